"""Parity checker for breadv2_b200 -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of ``bench.py`` may import this package.  Nothing in ``breadv2_b200``
imports it; the product path fails loudly when its CUDA library is missing
instead of falling back here.

Two CPU implementations live behind this module:

* ``liboracle.so`` -- ``oracle.c``, this repository's C restatement of the
  reference's CPU arithmetic (every function cites the reference file:line it
  restates);
* ``_ref/libbread_ref.so`` -- the reference's OWN CPU code (``layer_ops.cu``,
  ``dequant_q4k_cpu.c`` ...) compiled from its sources by ``oracle/Makefile``.
  It exists where the reference checkout was available at build time (it is
  built here and shipped as a git-ignored binary).

The restatement is pinned against the reference's known-answer blocks and
against fixtures produced by the compiled reference (``tests/golden``).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libbread_ref.so")
REF_GPU_SO = os.path.join(HERE, "_ref", "libbread_refgpu.so")

Q8_0, Q4_K, Q6_K = 8, 12, 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34}
BLOCK_ELEMS = {Q4_K: 256, Q6_K: 256, Q8_0: 32}

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float


def reference_source() -> str | None:
    """Where the reference checkout is: $BREAD_REF_SRC, else the
    ``reference_path`` recorded in the repository's BASELINE.json; None when
    neither names an existing directory (e.g. on a GPU box, which only uses
    the prebuilt _ref/ library)."""
    cand = os.environ.get("BREAD_REF_SRC")
    if not cand:
        try:
            import json

            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                cand = json.load(f).get("reference_path")
        except (OSError, ValueError):
            cand = None
    return cand if cand and os.path.isdir(cand) else None


def build(ref_src: str | None = None, verbose: bool = False) -> None:
    """Compile liboracle.so and, when the reference checkout exists, _ref/."""
    ref_src = ref_src or reference_source()
    targets = ["oracle"]
    cmd = ["make", "-s", "-C", HERE]
    if ref_src and os.path.isdir(ref_src):
        targets.append("ref")
        cmd.append(f"REF={ref_src}")
    cmd += targets
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")
    if verbose:
        print(out.stdout)


_lib = None
_ref = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_h2f.restype = _F
        L.orc_h2f.argtypes = [ctypes.c_uint16]
        L.orc_h2f_ftz.restype = _F
        L.orc_h2f_ftz.argtypes = [ctypes.c_uint16]
        L.orc_f2h.restype = ctypes.c_uint16
        L.orc_f2h.argtypes = [_F]
        L.orc_dequant.argtypes = [_P, _I, ctypes.c_longlong, _P, _I]
        L.orc_matvec_f32.argtypes = [_P, _I, _P, _P, _I, _I]
        L.orc_matvec_f64.argtypes = [_P, _I, _P, _P, _I, _I, _I]
        L.orc_route.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P]
        L.orc_router_logits_f64.argtypes = [_P, _P, _I, _I, _I, _P]
        L.orc_softmax.argtypes = [_P, _I]
        L.orc_topk.argtypes = [_P, _I, _I, _P, _P]
        L.orc_swiglu.argtypes = [_P, _P, _P, _I]
        L.orc_moe_f64.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.orc_moe_f32.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.orc_rmsnorm_f64.argtypes = [_P, _P, _I, ctypes.c_double]
        L.orc_synth_blocks.argtypes = [_P, ctypes.c_longlong, _I, ctypes.c_uint64, ctypes.c_uint64]
        L.orc_synth_normal.argtypes = [_P, ctypes.c_longlong, _F, ctypes.c_uint64, ctypes.c_uint64, _I]
        _lib = L
    return _lib


def synth_blocks(n_blocks: int, qtype: int, seed: int, stream_id: int) -> np.ndarray:
    """Seeded synthetic blocks, the same bytes as breadv2_b200.synth_blocks_host."""
    out = np.empty(n_blocks * BLOCK_BYTES[qtype], np.uint8)
    if lib().orc_synth_blocks(_p(out), n_blocks, qtype, seed, stream_id):
        raise ValueError(f"synth_blocks: bad qtype {qtype}")
    return out


def synth_normal(n: int, stddev: float, seed: int, stream_id: int, half: bool = False) -> np.ndarray:
    """Seeded N(0, stddev^2) values (fp32, or fp16 bits as uint16), the same as
    breadv2_b200.synth_normal_host."""
    out = np.empty(n, np.uint16 if half else np.float32)
    lib().orc_synth_normal(_p(out), n, stddev, seed, stream_id, 1 if half else 0)
    return out


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    """The reference's own CPU code (raises if it was never built)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} missing: build it with oracle.build() where the reference exists")
        L = ctypes.CDLL(REF_SO)
        for n in ("ref_dequant_q4k_block", "ref_dequant_q6k_block", "ref_dequant_q4k_block_ftz",
                  "ref_dequant_q6k_block_ftz"):
            getattr(L, n).argtypes = [_P, _P]
        L.ref_tensor_matvec.argtypes = [_P, ctypes.c_uint32, _P, _P, _I, _I]
        L.ref_swiglu.argtypes = [_P, _P, _P, _I]
        L.ref_softmax.argtypes = [_P, _I]
        L.ref_topk.argtypes = [_P, _I, _I, _P, _P]
        L.ref_sigmoid.restype = _F
        L.ref_sigmoid.argtypes = [_F]
        L.ref_route.argtypes = [_P, _P, _P, _I, _I, _I, _I, _P, _P, _P]
        L.ref_moe_block.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P]
        L.ref_kat.restype = _I
        L.ref_max_threads.restype = _I
        _ref = L
    return _ref


_refgpu = None


def refgpu_available() -> bool:
    return os.path.exists(REF_GPU_SO)


def refgpu() -> ctypes.CDLL:
    """The reference's own GPU GEMV (kernels.cu for sm_100a) with the
    expert_bench.cu launch loop (ref_gpu_shim.cu): measurement only."""
    global _refgpu
    if _refgpu is None:
        if not os.path.exists(REF_GPU_SO):
            raise FileNotFoundError(f"{REF_GPU_SO} missing: build it with oracle.build() where the reference exists")
        L = ctypes.CDLL(REF_GPU_SO)
        L.refgpu_matvec.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.refgpu_expert_loop.argtypes = [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I, _I, _P]
        _refgpu = L
    return _refgpu


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(_P)


# ---------------------------------------------------------------------------
# restatement (liboracle.so)
# ---------------------------------------------------------------------------

def h2f(bits: int) -> float:
    return lib().orc_h2f(bits)


def f2h_bits(x: float) -> int:
    return lib().orc_f2h(x)


def dequant(w: np.ndarray, qtype: int, n_blocks: int, ftz: bool = False) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    assert w.size >= n_blocks * BLOCK_BYTES[qtype]
    out = np.empty(n_blocks * BLOCK_ELEMS[qtype], dtype=np.float32)
    rc = lib().orc_dequant(_p(w), qtype, n_blocks, _p(out), int(ftz))
    assert rc == 0
    return out


def matvec_f32(w: np.ndarray, qtype: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    assert lib().orc_matvec_f32(_p(w), qtype, _p(x), _p(y), rows, cols) == 0
    return y


def matvec_f64(w: np.ndarray, qtype: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """x: [T, cols] or [cols] fp32 -> fp64 [T, rows] (or [rows])."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    squeeze = x.ndim == 1
    X = x.reshape(-1, cols)
    T = X.shape[0]
    y = np.empty((T, rows), dtype=np.float64)
    assert lib().orc_matvec_f64(_p(w), qtype, _p(X), _p(y), rows, cols, T) == 0
    return y[0] if squeeze else y


def route(x: np.ndarray, W_r: np.ndarray, w_sg_bits: np.ndarray | None, top_k: int):
    """x [T,H] fp32, W_r [E,H] fp32, w_sg_bits [H] uint16 or None.
    Returns idx [T,k] int32, w [T,k] fp32, sg_weight [T] fp32, logits [T,E] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    W_r = np.ascontiguousarray(W_r, dtype=np.float32)
    T, H = x.shape
    E = W_r.shape[0]
    idx = np.empty((T, top_k), dtype=np.int32)
    wt = np.empty((T, top_k), dtype=np.float32)
    sg = np.empty(T, dtype=np.float32)
    lg = np.empty((T, E), dtype=np.float32)
    sgp = None if w_sg_bits is None else _p(np.ascontiguousarray(w_sg_bits, dtype=np.uint16))
    assert lib().orc_route(_p(x), _p(W_r), sgp, T, H, E, top_k, _p(idx), _p(wt), _p(sg), _p(lg)) == 0
    return idx, wt, sg, lg


def router_logits_f64(x: np.ndarray, W_r: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    W_r = np.ascontiguousarray(W_r, dtype=np.float32)
    T, H = x.shape
    E = W_r.shape[0]
    out = np.empty((T, E), dtype=np.float64)
    lib().orc_router_logits_f64(_p(x), _p(W_r), T, H, E, _p(out))
    return out


def routing_margin(x: np.ndarray, W_r: np.ndarray, top_k: int) -> np.ndarray:
    """Per token: fp64 gap between the k-th and (k+1)-th largest logit, and the
    smallest gap among the chosen k (ties inside the top-k reorder weights)."""
    lg = router_logits_f64(x, W_r)
    s = -np.sort(-lg, axis=1)
    gaps = s[:, : top_k] - s[:, 1: top_k + 1]
    return gaps.min(axis=1)


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    o = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), _p(o), g.size)
    return o


class ExpertSet:
    """Host copies of a layer's expert weights, indexed by expert id."""

    def __init__(self, gate: list, up: list, down: list, sh_gate=None, sh_up=None, sh_down=None):
        self.gate = [np.ascontiguousarray(a, dtype=np.uint8) for a in gate]
        self.up = [np.ascontiguousarray(a, dtype=np.uint8) for a in up]
        self.down = [np.ascontiguousarray(a, dtype=np.uint8) for a in down]
        self.sh = None
        if sh_gate is not None:
            self.sh = tuple(np.ascontiguousarray(a, dtype=np.uint8) for a in (sh_gate, sh_up, sh_down))

    def _tables(self):
        n = len(self.gate)
        tab = []
        for lst in (self.gate, self.up, self.down):
            arr = (_P * n)(*[a.ctypes.data for a in lst])
            tab.append(arr)
        sh = (None, None, None) if self.sh is None else tuple(_p(a) for a in self.sh)
        return tab, sh


def moe_f64(es: ExpertSet, x, idx, wt, sg_weight, H: int, I: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H)
    T = x.shape[0]
    idx = np.ascontiguousarray(idx, dtype=np.int32).reshape(T, -1)
    top_k = idx.shape[1]
    wt = np.ascontiguousarray(wt, dtype=np.float32).reshape(T, top_k)
    sg = np.ascontiguousarray(sg_weight, dtype=np.float32).reshape(T)
    out = np.empty((T, H), dtype=np.float64)
    (tg, tu, td), (sgp, sup, sdp) = es._tables()
    rc = lib().orc_moe_f64(tg, tu, td, sgp, sup, sdp, _p(x), _p(idx), _p(wt), _p(sg), T, H, I, top_k, _p(out))
    assert rc == 0
    return out


def moe_f32(es: ExpertSet, x, idx, wt, sg_weight, H: int, I: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H)
    T = x.shape[0]
    idx = np.ascontiguousarray(idx, dtype=np.int32).reshape(T, -1)
    top_k = idx.shape[1]
    wt = np.ascontiguousarray(wt, dtype=np.float32).reshape(T, top_k)
    sg = np.ascontiguousarray(sg_weight, dtype=np.float32).reshape(T)
    out = np.empty((T, H), dtype=np.float32)
    (tg, tu, td), (sgp, sup, sdp) = es._tables()
    rc = lib().orc_moe_f32(tg, tu, td, sgp, sup, sdp, _p(x), _p(idx), _p(wt), _p(sg), T, H, I, top_k, _p(out))
    assert rc == 0
    return out


def rmsnorm_f64(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float64)
    y = np.empty_like(x)
    for t in range(x.shape[0]):
        lib().orc_rmsnorm_f64(_p(x[t]), _p(y[t]), x.shape[1], eps)
    return y


# ---------------------------------------------------------------------------
# the reference's own code (_ref/libbread_ref.so)
# ---------------------------------------------------------------------------

def ref_dequant(w: np.ndarray, qtype: int, n_blocks: int, ftz: bool = False) -> np.ndarray:
    R = ref()
    fn = {(Q4_K, False): R.ref_dequant_q4k_block, (Q6_K, False): R.ref_dequant_q6k_block,
          (Q4_K, True): R.ref_dequant_q4k_block_ftz, (Q6_K, True): R.ref_dequant_q6k_block_ftz}[(qtype, ftz)]
    w = np.ascontiguousarray(w, dtype=np.uint8)
    bb = BLOCK_BYTES[qtype]
    out = np.empty(n_blocks * 256, dtype=np.float32)
    base_w, base_o = w.ctypes.data, out.ctypes.data
    for b in range(n_blocks):
        fn(ctypes.c_void_p(base_w + b * bb), ctypes.c_void_p(base_o + b * 1024))
    return out


def ref_matvec(w: np.ndarray, qtype: int, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    ref().ref_tensor_matvec(_p(w), qtype, _p(x), _p(y), rows, cols)
    return y


def ref_route(x, W_r, w_sg_bits, top_k: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    W_r = np.ascontiguousarray(W_r, dtype=np.float32)
    T, H = x.shape
    E = W_r.shape[0]
    idx = np.empty((T, top_k), dtype=np.int32)
    wt = np.empty((T, top_k), dtype=np.float32)
    sg = np.empty(T, dtype=np.float32)
    sgp = None if w_sg_bits is None else _p(np.ascontiguousarray(w_sg_bits, dtype=np.uint16))
    ref().ref_route(_p(x), _p(W_r), sgp, T, H, E, top_k, _p(idx), _p(wt), _p(sg))
    return idx, wt, sg


def ref_softmax_topk(logits: np.ndarray, top_k: int):
    p = np.array(logits, dtype=np.float32, copy=True)
    ref().ref_softmax(_p(p), p.size)
    idx = np.empty(top_k, dtype=np.int32)
    wt = np.empty(top_k, dtype=np.float32)
    ref().ref_topk(_p(p), p.size, top_k, _p(idx), _p(wt))
    return p, idx, wt


def ref_swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    o = np.empty_like(g)
    ref().ref_swiglu(_p(g), _p(u), _p(o), g.size)
    return o


def ref_moe_block(es: ExpertSet, x, idx, wt, sg_weight, H: int, I: int, n_threads: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H)
    T = x.shape[0]
    idx = np.ascontiguousarray(idx, dtype=np.int32).reshape(T, -1)
    top_k = idx.shape[1]
    wt = np.ascontiguousarray(wt, dtype=np.float32).reshape(T, top_k)
    sg = np.ascontiguousarray(sg_weight, dtype=np.float32).reshape(T)
    out = np.empty((T, H), dtype=np.float32)
    (tg, tu, td), (sgp, sup, sdp) = es._tables()
    rc = ref().ref_moe_block(tg, tu, td, sgp, sup, sdp, _p(x), _p(idx), _p(wt), _p(sg), T, H, I, top_k,
                             n_threads, _p(out))
    assert rc == 0
    return out


class _RefGgufTensor(ctypes.Structure):
    # gguf_tensor_t, gguf.h:80-88
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
                ("dims", ctypes.c_uint64 * 4), ("offset", ctypes.c_uint64), ("size", ctypes.c_uint64),
                ("n_elems", ctypes.c_uint64)]


def ref_gguf_index(path: str) -> dict:
    """The reference's own parser (gguf_open, gguf.c:306-374, compiled into
    _ref/) on a well-formed file: version, data offset and every tensor info.
    (It exits the process on a malformed file, so only valid files go here.)"""
    L = ref()
    L.gguf_open.restype = ctypes.c_void_p
    L.gguf_open.argtypes = [ctypes.c_char_p]
    L.gguf_close.argtypes = [ctypes.c_void_p]
    L.gguf_version.restype = ctypes.c_uint32
    L.gguf_version.argtypes = [ctypes.c_void_p]
    L.gguf_num_tensors.restype = ctypes.c_uint64
    L.gguf_num_tensors.argtypes = [ctypes.c_void_p]
    L.gguf_data_offset.restype = ctypes.c_uint64
    L.gguf_data_offset.argtypes = [ctypes.c_void_p]
    L.gguf_tensor_by_idx.restype = ctypes.POINTER(_RefGgufTensor)
    L.gguf_tensor_by_idx.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    ctx = L.gguf_open(path.encode())
    assert ctx, "reference gguf_open failed"
    out = {"version": L.gguf_version(ctx), "data_offset": L.gguf_data_offset(ctx), "tensors": []}
    for i in range(L.gguf_num_tensors(ctx)):
        t = L.gguf_tensor_by_idx(ctx, i).contents
        out["tensors"].append({"name": t.name.decode(), "type": t.type, "dims": list(t.dims[: t.n_dims]),
                               "offset": t.offset, "size": t.size, "n_elems": t.n_elems})
    L.gguf_close(ctx)
    return out


def ref_kat() -> int:
    """Run the reference's own known-answer main() (dequant_q4k_cpu.c:177-288); 0 = PASS."""
    return ref().ref_kat()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))
