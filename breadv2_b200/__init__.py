"""breadv2_b200 -- sm_100a quantised-expert MoE path of the BREAD decode engine.

Host-side mirror of the reference's operator interface for this path, over the
C ABI of ``include/bread_b200.h`` (``libbread_b200.so``).  Device memory and
streams come from PyTorch; every computation runs in the CUDA library.

Reference interfaces mirrored (arahe-dev/breadv2):
  matvec            bread_matvec                kernels.cu:289-308
  rmsnorm_half ...  bread_rmsnorm_half etc.     layer_logic.cu:28-31
  moe_route         route_layer (on device)     one_layer.cu:937-992
  moe_ffn           MoE block of one layer      one_layer.cu:1820-1985
  ExpertStack       decode loop over layers     main.cu:677-713 (MoE part)
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import BreadError, StackConfig, check, device_error, last_error, lib  # noqa: F401

QTYPE_Q8_0, QTYPE_Q4_K, QTYPE_Q6_K = 8, 12, 14
BLOCK_BYTES = {QTYPE_Q4_K: 144, QTYPE_Q6_K: 210, QTYPE_Q8_0: 34}
BLOCK_ELEMS = {QTYPE_Q4_K: 256, QTYPE_Q6_K: 256, QTYPE_Q8_0: 32}


def _s(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _p(t) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    if isinstance(t, int):
        return ctypes.c_void_p(t)
    return ctypes.c_void_p(t.data_ptr())


def matrix_bytes(rows: int, cols: int, qtype: int) -> int:
    return rows * (cols // BLOCK_ELEMS[qtype]) * BLOCK_BYTES[qtype]


# ---- GEMV ----------------------------------------------------------------
def matvec(w, x, y, rows: int, cols: int, qtype: int, stream=None) -> None:
    """bread_matvec (kernels.cu:289): fp16 x [cols] -> fp16 y [rows]."""
    check(lib().bread_matvec_f16(_p(w), _p(x), _p(y), rows, cols, qtype, _s(stream)), "bread_matvec")


def matvec_f32(w, x, rows: int, cols: int, qtype: int, y=None, stream=None):
    """fp32 y = W x.  x: [cols] or [T, cols] (T <= 64) fp32 on the device."""
    T = 1 if x.dim() == 1 else x.shape[0]
    if y is None:
        y = torch.empty((rows,) if x.dim() == 1 else (T, rows), dtype=torch.float32, device=x.device)
    if T == 1:
        check(lib().bread_matvec_f32(_p(w), _p(x), _p(y), rows, cols, qtype, _s(stream)), "bread_matvec_f32")
    else:
        check(lib().bread_matvec_batch_f32(_p(w), _p(x), _p(y), rows, cols, qtype, T, _s(stream)),
              "bread_matvec_batch_f32")
    return y


def lm_head_argmax(w, x, rows: int, cols: int, qtype: int, round_half: bool = True, state=None, logits=None,
                   stream=None):
    """Greedy token of the head GEMV W x on the device (compute_logits +
    greedy_sample of main.cu:297-337): returns (token int32[1], value fp32[1])
    device tensors.  `state`: a reusable zeroed int64[2] device tensor."""
    import torch

    dev = x.device
    if state is None:
        state = torch.zeros(2, dtype=torch.int64, device=dev)
    token = torch.empty(1, dtype=torch.int32, device=dev)
    value = torch.empty(1, dtype=torch.float32, device=dev)
    check(lib().bread_lm_head_argmax(_p(w), _p(x), rows, cols, qtype, int(round_half),
                                     _p(logits) if logits is not None else None, _p(token), _p(value), _p(state),
                                     _s(stream)), "bread_lm_head_argmax")
    return token, value


def dequant(w, n_blocks: int, qtype: int, out=None, stream=None):
    """Bit-exact dequantisation (layer_ops.cu:44-105) of n_blocks blocks to fp32."""
    if out is None:
        out = torch.empty(n_blocks * BLOCK_ELEMS[qtype], dtype=torch.float32, device=w.device)
    check(lib().bread_dequant(_p(w), _p(out), n_blocks, qtype, _s(stream)), "bread_dequant")
    return out


# ---- fp16 glue (layer_logic.cu:28-31) --------------------------------------
def rmsnorm_half(x, w, eps: float, stream=None) -> None:
    check(lib().bread_rmsnorm_half_c(_p(x), _p(w), x.numel(), eps, _s(stream)), "bread_rmsnorm_half")


def silu_mul(gate, up, stream=None) -> None:
    check(lib().bread_silu_mul_c(_p(gate), _p(up), gate.numel(), _s(stream)), "bread_silu_mul")


def scale_accum(dst, src, scale: float, stream=None) -> None:
    check(lib().bread_scale_accum_c(_p(dst), _p(src), scale, dst.numel(), _s(stream)), "bread_scale_accum")


def copy_half(dst, src, stream=None) -> None:
    check(lib().bread_copy_half_c(_p(dst), _p(src), dst.numel(), _s(stream)), "bread_copy_half")


# ---- MoE block -------------------------------------------------------------
def workspace_bytes(T: int, H: int, I: int, E: int, top_k: int) -> int:
    return int(lib().bread_moe_workspace_bytes(T, H, I, E, top_k))


def alloc_workspace(T: int, H: int, I: int, E: int, top_k: int, device="cuda"):
    n = workspace_bytes(T, H, I, E, top_k)
    return torch.empty(n + 256, dtype=torch.uint8, device=device)


def _ws_ptr(ws):
    base = ws.data_ptr()
    return ctypes.c_void_p((base + 255) // 256 * 256), ws.numel() - ((base + 255) // 256 * 256 - base)


def moe_route(x, W_r, w_sg, top_k: int, workspace=None, stream=None):
    """route_layer (one_layer.cu:937-992) on the device for T tokens.
    x [T, H] fp32, W_r [E, H] fp32, w_sg [H] fp16 or None.
    Returns idx [T, k] int32, w [T, k] fp32, sg_weight [T] fp32."""
    T, H = x.shape
    E = W_r.shape[0]
    if workspace is None:
        workspace = alloc_workspace(T, H, 0, E, top_k, x.device)
    wp, wn = _ws_ptr(workspace)
    idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    sg = torch.empty(T, dtype=torch.float32, device=x.device)
    check(lib().bread_moe_route(_p(x), _p(W_r), _p(w_sg), T, H, E, top_k, _p(idx), _p(w), _p(sg), wp, wn,
                                _s(stream)), "bread_moe_route")
    return idx, w, sg


def pointer_table(tensors_or_ptrs, device="cuda"):
    """Device array of device pointers (the per-expert tables of loader.h:79-84)."""
    ptrs = [t if isinstance(t, int) else t.data_ptr() for t in tensors_or_ptrs]
    return torch.tensor(ptrs, dtype=torch.int64, device=device)


def moe_ffn(gate_tab, up_tab, down_tab, W_r, w_sg, shared, x, out, I: int, top_k: int, workspace=None,
            stream=None, want_routing: bool = False):
    """One layer's MoE FFN for T tokens: out += sum_k w_k expert_k(x) + sg * shared(x).
    *_tab: device int64 pointer tables [E]; shared: (gate, up, down) or None."""
    T, H = x.shape
    E = W_r.shape[0]
    if workspace is None:
        workspace = alloc_workspace(T, H, I, E, top_k, x.device)
    wp, wn = _ws_ptr(workspace)
    sh = (None, None, None) if shared is None else shared
    idx = w = sg = None
    if want_routing:
        idx = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
        sg = torch.empty(T, dtype=torch.float32, device=x.device)
    check(lib().bread_moe_ffn(_p(gate_tab), _p(up_tab), _p(down_tab), _p(W_r), _p(w_sg), _p(sh[0]), _p(sh[1]),
                              _p(sh[2]), _p(x), _p(out), T, H, I, E, top_k, _p(idx), _p(w), _p(sg), wp, wn,
                              _s(stream)), "bread_moe_ffn")
    return (idx, w, sg) if want_routing else None


# ---- GGUF model files -----------------------------------------------------------
class Gguf:
    """Tensor index of a GGUF v2/v3 file (bread_gguf_*; gguf.c:306-411)."""

    def __init__(self, path: str):
        h = ctypes.c_void_p(0)
        check(lib().bread_gguf_open(path.encode(), ctypes.byref(h)), "bread_gguf_open")
        self.handle = h

    def close(self):
        if self.handle:
            lib().bread_gguf_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        v, a = ctypes.c_uint32(0), ctypes.c_uint32(0)
        n, off = ctypes.c_uint64(0), ctypes.c_uint64(0)
        check(lib().bread_gguf_info(self.handle, ctypes.byref(v), ctypes.byref(n), ctypes.byref(a), ctypes.byref(off)),
              "bread_gguf_info")
        return {"version": v.value, "n_tensors": n.value, "alignment": a.value, "data_offset": off.value}

    @staticmethod
    def _dict(t) -> dict:
        return {"name": t.name.decode(), "type": t.type, "dims": list(t.dims[: t.n_dims]), "offset": t.offset,
                "size": t.size, "n_elems": t.n_elems}

    def tensor(self, index: int) -> dict:
        from ._lib import GgufTensor

        t = GgufTensor()
        check(lib().bread_gguf_tensor(self.handle, index, ctypes.byref(t)), "bread_gguf_tensor")
        return self._dict(t)

    def find(self, name: str):
        """Tensor info by exact name, or None when absent."""
        from ._lib import GgufTensor

        t = GgufTensor()
        if lib().bread_gguf_find(self.handle, name.encode(), ctypes.byref(t)) != 0:
            return None
        return self._dict(t)

    def read(self, offset: int, nbytes: int):
        import numpy as np

        out = np.empty(nbytes, dtype=np.uint8)
        check(lib().bread_gguf_read(self.handle, offset, out.ctypes.data_as(ctypes.c_void_p), nbytes), "bread_gguf_read")
        return out


# ---- expert stack ------------------------------------------------------------
class ExpertStack:
    """All layers' experts resident on this GPU (or this rank's share of them),
    synthetic weights from a seed; ``step`` runs one decode step."""

    def __init__(self, n_layers=40, hidden=2048, inter=512, n_experts=256, top_k=8, max_tokens=64,
                 shared_expert=True, norm_eps=1e-6, seed=1234, rank=0, world=1, norm_weight=True):
        self.cfg = StackConfig(n_layers, hidden, inter, n_experts, top_k, max_tokens, int(shared_expert), norm_eps,
                               seed, rank, world, int(norm_weight))
        h = ctypes.c_void_p(0)
        self.handle = None
        self._opened = []
        check(lib().bread_stack_create(ctypes.byref(h), ctypes.byref(self.cfg)), "bread_stack_create")
        self.handle = h

    @classmethod
    def from_gguf(cls, path: str, n_layers: int, top_k: int = 8, max_tokens: int = 64, norm_eps: float = 1e-6,
                  rank: int = 0, world: int = 1):
        """The stack of a GGUF model file's first n_layers MoE layers
        (bread_stack_create_gguf): shapes, shared expert and norm weights
        come from the file."""
        self = cls.__new__(cls)
        self.cfg = StackConfig(n_layers, 0, 0, 0, top_k, max_tokens, 0, norm_eps, 0, rank, world, 0)
        self.handle = None
        self._opened = []
        h = ctypes.c_void_p(0)
        check(lib().bread_stack_create_gguf(ctypes.byref(h), path.encode(), ctypes.byref(self.cfg)),
              "bread_stack_create_gguf")
        self.handle = h
        check(lib().bread_stack_get_config(h, ctypes.byref(self.cfg)), "bread_stack_get_config")
        return self

    def close(self):
        if self.handle:
            lib().bread_stack_destroy(self.handle)
            self.handle = None
        for p in self._opened:
            lib().bread_ipc_close_handle(ctypes.c_void_p(p))
        self._opened = []

    def mailbox(self):
        ptr, n = ctypes.c_void_p(0), ctypes.c_size_t(0)
        check(lib().bread_stack_mailbox(self.handle, ctypes.byref(ptr), ctypes.byref(n)), "bread_stack_mailbox")
        return ptr.value or 0, n.value

    def connect_peers(self, dist, group=None) -> None:
        """Expert parallel set-up: exchange CUDA IPC handles of every rank's
        mailbox over `dist` (torch.distributed, any backend) and map the peers'."""
        rank, world = self.cfg.rank, self.cfg.world
        ptr, _ = self.mailbox()
        handle = ctypes.create_string_buffer(64)
        check(lib().bread_ipc_get_handle(ctypes.c_void_p(ptr), handle), "bread_ipc_get_handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        peers = []
        for r, hb in enumerate(handles):
            if r == rank:
                peers.append(ptr)
                continue
            p = ctypes.c_void_p(0)
            buf = ctypes.create_string_buffer(bytes(hb), 64)
            check(lib().bread_ipc_open_handle(buf, ctypes.byref(p)), "bread_ipc_open_handle")
            self._opened.append(p.value)
            peers.append(p.value)
        arr = (ctypes.c_void_p * world)(*peers)
        check(lib().bread_stack_set_peers(self.handle, arr, world), "bread_stack_set_peers")

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return int(lib().bread_stack_device_bytes(self.handle))

    def launches_per_step(self, T: int) -> int:
        return int(lib().bread_stack_launches_per_step(self.handle, T))

    def layer(self, l: int) -> dict:
        ptrs = [ctypes.c_void_p(0) for _ in range(8)]
        lo, hi = ctypes.c_int(0), ctypes.c_int(0)
        check(lib().bread_stack_layer(self.handle, l, *[ctypes.byref(p) for p in ptrs], ctypes.byref(lo),
                                      ctypes.byref(hi)), "bread_stack_layer")
        keys = ["gate", "up", "down", "W_r", "w_sg", "sh_gate", "sh_up", "sh_down"]
        d = {k: (p.value or 0) for k, p in zip(keys, ptrs)}
        d["lo"], d["hi"] = lo.value, hi.value
        return d

    def norm_weight(self, l: int):
        """Layer l's pre-MoE RMSNorm weight (host fp32 [hidden]), or None for
        unit weight."""
        import numpy as np

        out = np.zeros(self.cfg.hidden, dtype=np.float32)
        has = ctypes.c_int(0)
        check(lib().bread_stack_norm_weight(self.handle, l, out.ctypes.data_as(ctypes.c_void_p), ctypes.byref(has)),
              "bread_stack_norm_weight")
        return out if has.value else None

    def step(self, h, stream=None) -> None:
        """h: [T, hidden] fp32 on this device, updated in place."""
        check(lib().bread_stack_step(self.handle, _p(h), h.shape[0], _s(stream)), "bread_stack_step")

    def profile_step(self, h, stream=None):
        """One instrumented step; returns per-layer (route, gate/up, down, combine) ms."""
        import numpy as np

        L = self.cfg.n_layers
        out = np.zeros(4 * L, dtype=np.float32)
        check(lib().bread_stack_profile_step(self.handle, _p(h), h.shape[0], _s(stream),
                                             out.ctypes.data_as(ctypes.c_void_p)), "bread_stack_profile_step")
        return out.reshape(L, 4)

    def profile_stamps(self):
        """Timestamps (ns) of the last profile_step: array [layers, ctas, 24] of
        the phase points listed in bread_stack_profile_stamps."""
        import numpy as np

        L = self.cfg.n_layers
        n = L * 1024 * 24
        buf = np.zeros(n, dtype=np.uint64)
        ctas = ctypes.c_int(0)
        check(lib().bread_stack_profile_stamps(self.handle, buf.ctypes.data_as(ctypes.c_void_p), n, ctypes.byref(ctas)),
              "bread_stack_profile_stamps")
        return buf[: L * ctas.value * 24].reshape(L, ctas.value, 24)

    def routing_stats(self):
        """Per layer of the last step: (expert groups computed here, token-expert pairs)."""
        import numpy as np

        L = self.cfg.n_layers
        g = np.zeros(L, dtype=np.int32)
        p = np.zeros(L, dtype=np.int32)
        check(lib().bread_stack_routing_stats(self.handle, g.ctypes.data_as(ctypes.c_void_p),
                                              p.ctypes.data_as(ctypes.c_void_p)), "bread_stack_routing_stats")
        return g, p

    def routing(self):
        """Routing of every layer of the last step as the kernel ran it:
        (idx [L, T, K] int32, w [L, T, K] fp32, sg_weight [L, T] fp32)."""
        import numpy as np

        L, K, Tm = self.cfg.n_layers, self.cfg.top_k, self.cfg.max_tokens
        idx = np.zeros(L * Tm * K, dtype=np.int32)
        w = np.zeros(L * Tm * K, dtype=np.float32)
        sg = np.zeros(L * Tm, dtype=np.float32)
        T = ctypes.c_int(0)
        check(lib().bread_stack_routing(self.handle, idx.ctypes.data_as(ctypes.c_void_p),
                                        w.ctypes.data_as(ctypes.c_void_p), sg.ctypes.data_as(ctypes.c_void_p),
                                        ctypes.byref(T)), "bread_stack_routing")
        T = T.value
        return (idx[: L * T * K].reshape(L, T, K), w[: L * T * K].reshape(L, T, K), sg[: L * T].reshape(L, T))

    def step_host(self, h_in, h_out, stream=None) -> None:
        """h_in/h_out: [T, hidden] fp32 host tensors (pinned for speed)."""
        check(lib().bread_stack_step_host(self.handle, _p(h_in), _p(h_out), h_in.shape[0], _s(stream)),
              "bread_stack_step_host")


# ---- synthetic data ----------------------------------------------------------
def synth_blocks(n_blocks: int, qtype: int, seed: int, stream_id: int, device="cuda", stream=None):
    out = torch.empty(n_blocks * BLOCK_BYTES[qtype], dtype=torch.uint8, device=device)
    check(lib().bread_synth_blocks(_p(out), n_blocks, qtype, seed, stream_id, _s(stream)), "bread_synth_blocks")
    return out


def synth_blocks_host(n_blocks: int, qtype: int, seed: int, stream_id: int):
    import numpy as np
    out = np.empty(n_blocks * BLOCK_BYTES[qtype], dtype=np.uint8)
    check(lib().bread_synth_blocks_host(out.ctypes.data_as(ctypes.c_void_p), n_blocks, qtype, seed, stream_id),
          "bread_synth_blocks_host")
    return out


def synth_normal_host(n: int, stddev: float, seed: int, stream_id: int, half: bool = False):
    import numpy as np
    out = np.empty(n, dtype=np.uint16 if half else np.float32)
    fn = lib().bread_synth_normal_f16_host if half else lib().bread_synth_normal_f32_host
    check(fn(out.ctypes.data_as(ctypes.c_void_p), n, stddev, seed, stream_id), "bread_synth_normal_host")
    return out


def synth_normal(n: int, stddev: float, seed: int, stream_id: int, half: bool = False, device="cuda", stream=None):
    out = torch.empty(n, dtype=torch.float16 if half else torch.float32, device=device)
    fn = lib().bread_synth_normal_f16 if half else lib().bread_synth_normal_f32
    check(fn(_p(out), n, stddev, seed, stream_id, _s(stream)), "bread_synth_normal")
    return out
