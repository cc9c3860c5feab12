"""ctypes binding of libstreamlx_cuda.so (include/streamlx_cuda.h).

The product path has no CPU fallback: if the shared object is missing or a
call fails, an exception is raised.  Tensors passed here must be CUDA tensors
(except the host arrays of ``copy_many``).
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libstreamlx_cuda.so")

SLX_OK = 0
ERRORS = {
    -1: "SLX_ERR_INVALID", -2: "SLX_ERR_UNSUPPORTED", -3: "SLX_ERR_CUDA",
    -4: "SLX_ERR_OUT_OF_RANGE", -5: "SLX_ERR_UNMAPPED_EXPERT",
    -6: "SLX_ERR_DEVICE_TIMEOUT", -7: "SLX_ERR_SCRATCH", -8: "SLX_ERR_IO",
    -9: "SLX_ERR_RANGE",
}
SLX_ERR_RANGE = -9
GEMV_GLU, GEMV_LINEAR = 0, 1

# every symbol the header declares (the CPU test checks they are exported)
EXPORTS = (
    "slx_version", "slx_last_error_string", "slx_expert_tiled_bytes",
    "slx_dense_tiled_bytes", "slx_pack_experts", "slx_pack_dense",
    "slx_switchglu_scratch_bytes",
    "slx_switchglu", "slx_qlinear", "slx_dequant_rows",
    "slx_router_scratch_bytes", "slx_router_topk", "slx_add_rmsnorm",
    "slx_qk_norm_rope_cache", "slx_attn_decode", "slx_attn_rope_decode",
    "slx_router_topk_multi_norm",
    "slx_argmax",
    "slx_copy_many", "slx_router_topk_noalloc", "slx_add_rmsnorm_out",
    "slx_event_record_external", "slx_event_elapsed_many",
    "slx_router_topk_multi", "slx_set_pdl", "slx_pread_many",
    "slx_set_switchglu_fused", "slx_switchglu_last_kernels",
    "slx_prefill_scratch_bytes", "slx_prefill_grouped",
    "slx_switchglu_serviced", "slx_host_device_ptr",
    "slx_ep_grid", "slx_switchglu_ep", "slx_ep_combine_rmsnorm",
    "slx_ipc_handle", "slx_ipc_open", "slx_ipc_close",
)
EP_MAX_RANKS = 8

# slx_fill_service layout constants (include/streamlx_cuda.h)
FILL_LOG_WORDS = 64
FILL_MAX_K = 16
FILL_HEADER_BYTES = 32
FILL_ITEM_BYTES = 80


class slx_qmat(C.Structure):
    _fields_ = [("weight", C.c_void_p), ("scales", C.c_void_p),
                ("biases", C.c_void_p)]


class slx_expert_bank(C.Structure):
    _fields_ = [("base", C.c_void_p), ("slot_stride", C.c_int64),
                ("n_slots", C.c_int32), ("hidden", C.c_int32),
                ("inter", C.c_int32), ("bits", C.c_int32)]


class slx_shared_expert(C.Structure):
    _fields_ = [("base", C.c_void_p), ("inter", C.c_int32)]


class SlxError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} failed: {ERRORS.get(rc, rc)}: {msg}")
        self.rc = rc


_lib = None

# Number of kernel launches issued through this binding (the bench reports
# the launches inside its timed region).  slx_switchglu launches two kernels.
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


class slx_fill_service(C.Structure):
    _fields_ = [("layer", C.c_int32), ("max_items", C.c_int32),
                ("stamp", C.c_void_p), ("log", C.c_void_p),
                ("pred_ids", C.c_void_p), ("pred_scores", C.c_void_p),
                ("park", C.c_void_p), ("release", C.c_void_p),
                ("desc", C.c_void_p), ("go", C.c_void_p),
                ("wait_ns", C.c_int64)]


class slx_ep_exchange(C.Structure):
    _fields_ = [("rank", C.c_int32), ("n_ranks", C.c_int32),
                ("layer", C.c_int32), ("n_layers", C.c_int32),
                ("stamp", C.c_void_p),
                ("recv", C.c_void_p * 8), ("count", C.c_void_p * 8),
                ("grid", C.c_int32), ("wait_ns", C.c_int64)]


class slx_router_head(C.Structure):
    _fields_ = [("w_gate", C.c_void_p), ("bias", C.c_void_p),
                ("ratio", C.c_void_p), ("force", C.c_void_p),
                ("forced_ids", C.c_void_p), ("out_ids", C.c_void_p),
                ("out_scores", C.c_void_p), ("scratch", C.c_void_p),
                ("scratch_bytes", C.c_size_t)]


def lib() -> C.CDLL:
    """Load the shared object (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with "
                "`python -m streamlx_b200.build` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        vp, i32, sz = C.c_void_p, C.c_int, C.c_size_t
        L.slx_version.restype = i32
        L.slx_set_pdl.restype = i32
        L.slx_set_pdl.argtypes = [i32]
        L.slx_set_switchglu_fused.restype = i32
        L.slx_set_switchglu_fused.argtypes = [i32]
        L.slx_switchglu_last_kernels.restype = i32
        L.slx_last_error_string.restype = C.c_char_p
        L.slx_expert_tiled_bytes.restype = sz
        L.slx_expert_tiled_bytes.argtypes = [i32, i32, i32]
        L.slx_dense_tiled_bytes.restype = sz
        L.slx_dense_tiled_bytes.argtypes = [i32, i32, i32]
        L.slx_pack_experts.restype = i32
        L.slx_pack_experts.argtypes = [C.POINTER(slx_qmat), C.POINTER(slx_qmat),
                                       C.POINTER(slx_qmat), i32, i32, i32,
                                       i32, vp, vp]
        L.slx_pack_dense.restype = i32
        L.slx_pack_dense.argtypes = [C.POINTER(slx_qmat), i32, i32, i32, vp, vp]
        L.slx_switchglu_scratch_bytes.restype = sz
        L.slx_switchglu_scratch_bytes.argtypes = [i32, i32, i32, i32]
        L.slx_switchglu.restype = i32
        L.slx_switchglu.argtypes = [C.POINTER(slx_expert_bank),
                                    C.POINTER(slx_shared_expert), vp, i32,
                                    i32, vp, vp, vp, i32, vp, vp, sz, vp, vp]
        L.slx_qlinear.restype = i32
        L.slx_qlinear.argtypes = [vp, i32, i32, i32, vp, i32, vp, vp, vp]
        L.slx_dequant_rows.restype = i32
        L.slx_dequant_rows.argtypes = [C.POINTER(slx_qmat), i32, i32, i32, vp,
                                       i32, i32, vp, i32, vp, vp]
        L.slx_router_scratch_bytes.restype = sz
        L.slx_router_scratch_bytes.argtypes = [i32, i32]
        L.slx_router_topk.restype = i32
        L.slx_router_topk.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                      vp, vp, vp, vp, vp, sz, vp, vp]
        L.slx_router_topk_multi.restype = i32
        L.slx_router_topk_multi.argtypes = [C.POINTER(slx_router_head), i32,
                                            vp, i32, i32, i32, i32, i32, vp,
                                            vp]
        L.slx_router_topk_multi_norm.restype = i32
        L.slx_router_topk_multi_norm.argtypes = [
            C.POINTER(slx_router_head), i32, vp, vp, vp, C.c_float, vp, vp,
            i32, i32, i32, i32, vp, vp]
        L.slx_router_topk_noalloc.restype = i32
        L.slx_router_topk_noalloc.argtypes = [vp, vp, vp, vp, i32, i32, i32,
                                              i32, i32, vp, vp, vp, vp, vp, vp]
        L.slx_add_rmsnorm.restype = i32
        L.slx_add_rmsnorm.argtypes = [vp, vp, vp, i32, i32, C.c_float, vp, vp]
        L.slx_add_rmsnorm_out.restype = i32
        L.slx_add_rmsnorm_out.argtypes = [vp, vp, vp, i32, i32, C.c_float, vp,
                                          vp, vp]
        L.slx_event_record_external.restype = i32
        L.slx_event_record_external.argtypes = [vp, vp]
        L.slx_event_elapsed_many.restype = i32
        L.slx_event_elapsed_many.argtypes = [C.POINTER(vp), C.POINTER(vp), i32,
                                             C.POINTER(C.c_float)]
        L.slx_qk_norm_rope_cache.restype = i32
        L.slx_qk_norm_rope_cache.argtypes = [vp, i32, i32, i32, i32, vp, vp,
                                             C.c_float, vp, vp, i32, vp, vp,
                                             vp, vp]
        L.slx_attn_rope_decode.restype = i32
        L.slx_attn_rope_decode.argtypes = [vp, i32, i32, i32, vp, vp,
                                           C.c_float, vp, vp, i32, vp, vp,
                                           vp, vp, vp]
        L.slx_attn_decode.restype = i32
        L.slx_attn_decode.argtypes = [vp, i32, i32, i32, i32, vp, vp, vp, i32,
                                      vp, vp]
        L.slx_argmax.restype = i32
        L.slx_argmax.argtypes = [vp, i32, i32, vp, vp]
        L.slx_pread_many.restype = i32
        L.slx_pread_many.argtypes = [vp, vp, vp, vp, i32, i32,
                                     C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.slx_copy_many.restype = i32
        L.slx_copy_many.argtypes = [vp, vp, vp, i32, vp]
        L.slx_prefill_scratch_bytes.restype = sz
        L.slx_prefill_scratch_bytes.argtypes = [i32, i32, i32, i32]
        L.slx_switchglu_serviced.restype = i32
        L.slx_switchglu_serviced.argtypes = [
            C.POINTER(slx_expert_bank), C.POINTER(slx_shared_expert), vp,
            i32, vp, vp, vp, i32, vp, vp, sz, vp,
            C.POINTER(slx_fill_service), vp]
        L.slx_ep_grid.restype = i32
        L.slx_switchglu_ep.restype = i32
        L.slx_switchglu_ep.argtypes = [
            C.POINTER(slx_expert_bank), C.POINTER(slx_shared_expert), vp,
            i32, vp, vp, vp, i32, vp, sz, vp, C.POINTER(slx_ep_exchange), vp]
        L.slx_ep_combine_rmsnorm.restype = i32
        L.slx_ep_combine_rmsnorm.argtypes = [
            C.POINTER(slx_ep_exchange), vp, i32, i32, i32, vp, vp, C.c_float,
            vp, vp, vp, vp]
        L.slx_ipc_handle.restype = i32
        L.slx_ipc_handle.argtypes = [vp, vp, C.POINTER(C.c_int64)]
        L.slx_ipc_open.restype = i32
        L.slx_ipc_open.argtypes = [vp, C.POINTER(vp)]
        L.slx_ipc_close.restype = i32
        L.slx_ipc_close.argtypes = [vp]
        L.slx_host_device_ptr.restype = i32
        L.slx_host_device_ptr.argtypes = [vp, C.POINTER(vp)]
        L.slx_prefill_grouped.restype = i32
        L.slx_prefill_grouped.argtypes = [C.POINTER(slx_expert_bank), vp, i32,
                                          vp, i32, vp, i32, vp, vp, i32, vp,
                                          sz, vp, vp]
        _lib = L
    return _lib


def set_pdl(on: bool) -> bool:
    """Programmatic dependent launch for this thread's next launches;
    returns the previous setting."""
    return bool(lib().slx_set_pdl(1 if on else 0))


def set_switchglu_fused(on: bool) -> bool:
    """Decode SwitchGLU as one cooperative launch (default) or two."""
    return bool(lib().slx_set_switchglu_fused(1 if on else 0))


def _check(fn: str, rc: int) -> None:
    if rc != SLX_OK:
        raise SlxError(fn, rc, lib().slx_last_error_string().decode())


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def qmat(w: torch.Tensor, s: torch.Tensor, b: torch.Tensor) -> slx_qmat:
    return slx_qmat(w.data_ptr(), s.data_ptr(), b.data_ptr())


def expert_tiled_bytes(hidden: int, inter: int, bits: int) -> int:
    return int(lib().slx_expert_tiled_bytes(hidden, inter, bits))


def dense_tiled_bytes(out_features: int, in_features: int, bits: int) -> int:
    return int(lib().slx_dense_tiled_bytes(out_features, in_features, bits))


def slot_stride(hidden: int, inter: int, bits: int) -> int:
    """Bytes between pool slots: the tiled expert size rounded to 256."""
    n = expert_tiled_bytes(hidden, inter, bits)
    return (n + 255) // 256 * 256


def pack_experts(experts: list, hidden: int, inter: int, bits: int,
                 dst_ptrs: list[int],
                 stream: torch.cuda.Stream | None = None) -> None:
    """experts: list of (gate3, up3, down3), each a (weight, scales, biases)
    tuple of CUDA tensors in the MLX layout; dst_ptrs: device addresses."""
    n = len(experts)
    if n == 0:
        return
    G = (slx_qmat * n)(*[qmat(*e[0]) for e in experts])
    U = (slx_qmat * n)(*[qmat(*e[1]) for e in experts])
    D = (slx_qmat * n)(*[qmat(*e[2]) for e in experts])
    P = (C.c_void_p * n)(*dst_ptrs)
    rc = lib().slx_pack_experts(G, U, D, n, hidden, inter, bits, P,
                                stream_ptr(stream))
    _check("slx_pack_experts", rc)
    _count(1)


def pack_dense(w3, out_features: int, in_features: int, bits: int,
               dst: torch.Tensor, stream: torch.cuda.Stream | None = None
               ) -> None:
    m = qmat(*w3)
    rc = lib().slx_pack_dense(C.byref(m), out_features, in_features, bits,
                              dst.data_ptr(), stream_ptr(stream))
    _check("slx_pack_dense", rc)
    _count(1)


def bank_struct(pool: torch.Tensor, n_slots: int, hidden: int, inter: int,
                bits: int, stride: int | None = None) -> slx_expert_bank:
    """pool: uint8 CUDA tensor holding n_slots tiled experts."""
    st = stride if stride is not None else slot_stride(hidden, inter, bits)
    return slx_expert_bank(pool.data_ptr(), st, n_slots, hidden, inter, bits)


def shared_struct(buf: torch.Tensor, inter: int) -> slx_shared_expert:
    return slx_shared_expert(buf.data_ptr(), inter)


def switchglu_scratch_bytes(T: int, k: int, inter: int, shared_inter: int = 0
                            ) -> int:
    return int(lib().slx_switchglu_scratch_bytes(T, k, inter, shared_inter))


def switchglu(bank: slx_expert_bank, x: torch.Tensor, ids: torch.Tensor,
              out: torch.Tensor, scratch: torch.Tensor, status: torch.Tensor,
              scores: torch.Tensor | None = None,
              slot_table: torch.Tensor | None = None,
              shared: slx_shared_expert | None = None,
              stream: torch.cuda.Stream | None = None) -> None:
    T, k = ids.shape[-2], ids.shape[-1]
    rc = lib().slx_switchglu(
        C.byref(bank), C.byref(shared) if shared is not None else None,
        x.data_ptr(), T, k, ids.data_ptr(), ptr(scores), ptr(slot_table),
        int(slot_table.numel()) if slot_table is not None else 0,
        out.data_ptr(), scratch.data_ptr(), scratch.numel() * scratch.element_size(),
        status.data_ptr(), stream_ptr(stream))
    _check("slx_switchglu", rc)
    _count(lib().slx_switchglu_last_kernels())


def switchglu_serviced(bank: slx_expert_bank, x: torch.Tensor,
                       ids: torch.Tensor, scores: torch.Tensor,
                       slot_table: torch.Tensor, out: torch.Tensor,
                       scratch: torch.Tensor, status: torch.Tensor,
                       svc: slx_fill_service,
                       shared: slx_shared_expert | None = None,
                       stream: torch.cuda.Stream | None = None) -> None:
    """One decode token's SwitchGLU with the in-kernel slot fill."""
    k = ids.shape[-1]
    rc = lib().slx_switchglu_serviced(
        C.byref(bank), C.byref(shared) if shared is not None else None,
        x.data_ptr(), k, ids.data_ptr(), scores.data_ptr(),
        slot_table.data_ptr(), int(slot_table.numel()), out.data_ptr(),
        scratch.data_ptr(), scratch.numel() * scratch.element_size(),
        status.data_ptr(), C.byref(svc), stream_ptr(stream))
    _check("slx_switchglu_serviced", rc)
    _count(1)


def ep_grid() -> int:
    n = int(lib().slx_ep_grid())
    if n <= 0:
        _check("slx_ep_grid", n)
    return n


def switchglu_ep(bank, x, ids, scores, slot_table, scratch, status, ep,
                 shared=None, stream=None) -> None:
    """One decode token's SwitchGLU in expert-parallel mode."""
    k = ids.shape[-1]
    rc = lib().slx_switchglu_ep(
        C.byref(bank), C.byref(shared) if shared is not None else None,
        x.data_ptr(), k, ids.data_ptr(), scores.data_ptr(),
        slot_table.data_ptr(), int(slot_table.numel()), scratch.data_ptr(),
        scratch.numel() * scratch.element_size(), status.data_ptr(),
        C.byref(ep), stream_ptr(stream))
    _check("slx_switchglu_ep", rc)
    _count(1)


def ep_combine_rmsnorm(ep, scores, k: int, hidden: int, has_shared: bool,
                       h_in, weight, eps: float, h_out, y, status,
                       stream=None) -> None:
    rc = lib().slx_ep_combine_rmsnorm(
        C.byref(ep), scores.data_ptr(), k, hidden, 1 if has_shared else 0,
        h_in.data_ptr(), weight.data_ptr(), eps, h_out.data_ptr(),
        y.data_ptr(), status.data_ptr(), stream_ptr(stream))
    _check("slx_ep_combine_rmsnorm", rc)
    _count(1)


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding t, t's offset)."""
    buf = (C.c_char * 64)()
    off = C.c_int64(0)
    rc = lib().slx_ipc_handle(t.data_ptr(), buf, C.byref(off))
    _check("slx_ipc_handle", rc)
    return bytes(buf), int(off.value)


def ipc_open(handle: bytes) -> int:
    out = C.c_void_p()
    buf = (C.c_char * 64).from_buffer_copy(handle)
    rc = lib().slx_ipc_open(buf, C.byref(out))
    _check("slx_ipc_open", rc)
    return int(out.value)


def ipc_close(base: int) -> None:
    _check("slx_ipc_close", lib().slx_ipc_close(base))


def host_device_ptr(host_ptr: int) -> int:
    """Device address of page-locked host memory."""
    out = C.c_void_p()
    rc = lib().slx_host_device_ptr(host_ptr, C.byref(out))
    _check("slx_host_device_ptr", rc)
    return int(out.value or 0)


def qlinear(w_tiled: torch.Tensor, out_features: int, in_features: int,
            bits: int, x: torch.Tensor, y: torch.Tensor, status: torch.Tensor,
            T: int | None = None,
            stream: torch.cuda.Stream | None = None) -> None:
    rc = lib().slx_qlinear(w_tiled.data_ptr(), out_features, in_features, bits,
                           x.data_ptr(), T if T is not None else x.shape[0],
                           y.data_ptr(), status.data_ptr(), stream_ptr(stream))
    _check("slx_qlinear", rc)
    _count(1)


def dequant_rows(w3, in_features: int, bits: int, rows: torch.Tensor | None,
                 nrows: int, n_src_rows: int, out: torch.Tensor,
                 status: torch.Tensor, group_size: int = 64,
                 stream: torch.cuda.Stream | None = None) -> None:
    m = qmat(*w3)
    rc = lib().slx_dequant_rows(C.byref(m), in_features, bits, group_size,
                                ptr(rows), nrows, n_src_rows, out.data_ptr(),
                                1 if out.dtype == torch.bfloat16 else 0,
                                status.data_ptr(), stream_ptr(stream))
    _check("slx_dequant_rows", rc)
    _count(1)


def router_scratch_bytes(T: int, E: int) -> int:
    return int(lib().slx_router_scratch_bytes(T, E))


def router_topk(x: torch.Tensor, w_gate: torch.Tensor, bias, k: int,
                norm_topk: bool, out_ids: torch.Tensor,
                out_scores: torch.Tensor, scratch: torch.Tensor,
                status: torch.Tensor, ratio: torch.Tensor | None = None,
                force: torch.Tensor | None = None,
                forced_ids: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> None:
    T, H = x.shape[-2], x.shape[-1]
    E = w_gate.shape[0]
    rc = lib().slx_router_topk(
        x.data_ptr(), ptr(ratio), w_gate.data_ptr(), ptr(bias), T, H, E, k,
        1 if norm_topk else 0, ptr(force), ptr(forced_ids), out_ids.data_ptr(),
        out_scores.data_ptr(), scratch.data_ptr(),
        scratch.numel() * scratch.element_size(), status.data_ptr(),
        stream_ptr(stream))
    _check("slx_router_topk", rc)
    _count(1)


def router_head(w_gate, bias, out_ids, out_scores, scratch, ratio=None,
                force=None, forced_ids=None) -> slx_router_head:
    return slx_router_head(w_gate.data_ptr(), ptr(bias), ptr(ratio),
                           ptr(force), ptr(forced_ids), out_ids.data_ptr(),
                           out_scores.data_ptr(), scratch.data_ptr(),
                           scratch.numel() * scratch.element_size())


def router_topk_multi(x: torch.Tensor, heads: list, E: int, k: int,
                      norm_topk: bool, status: torch.Tensor,
                      stream=None) -> None:
    """One launch of 1-2 router heads (router_head structs) over x [T, H]."""
    T, H = x.shape[-2], x.shape[-1]
    arr = (slx_router_head * len(heads))(*heads)
    rc = lib().slx_router_topk_multi(arr, len(heads), x.data_ptr(), T, H, E,
                                     k, 1 if norm_topk else 0,
                                     status.data_ptr(), stream_ptr(stream))
    _check("slx_router_topk_multi", rc)
    _count(1)


def router_topk_multi_norm(heads: list, h_in, delta, norm_weight, eps: float,
                           h_out, x_out, E: int, k: int, norm_topk: bool,
                           status: torch.Tensor, stream=None) -> None:
    """One decode token: h_out = h_in + delta, x_out = RMSNorm(h_out) * w,
    and 1-2 router heads on x_out, in one launch."""
    H = h_in.shape[-1]
    arr = (slx_router_head * len(heads))(*heads)
    rc = lib().slx_router_topk_multi_norm(
        arr, len(heads), h_in.data_ptr(), ptr(delta), norm_weight.data_ptr(),
        eps, h_out.data_ptr(), x_out.data_ptr(), H, E, k,
        1 if norm_topk else 0, status.data_ptr(), stream_ptr(stream))
    _check("slx_router_topk_multi_norm", rc)
    _count(1)


def add_rmsnorm(h, delta, weight, eps: float, y, stream=None) -> None:
    T, H = h.shape[-2], h.shape[-1]
    rc = lib().slx_add_rmsnorm(h.data_ptr(), ptr(delta), weight.data_ptr(), T,
                               H, eps, y.data_ptr(), stream_ptr(stream))
    _check("slx_add_rmsnorm", rc)
    _count(1)


def add_rmsnorm_out(h_in, delta, weight, eps: float, h_out, y,
                    stream=None) -> None:
    T, H = h_in.shape[-2], h_in.shape[-1]
    rc = lib().slx_add_rmsnorm_out(h_in.data_ptr(), ptr(delta),
                                   weight.data_ptr(), T, H, eps,
                                   h_out.data_ptr(), y.data_ptr(),
                                   stream_ptr(stream))
    _check("slx_add_rmsnorm_out", rc)
    _count(1)


def event_record_external(event: torch.cuda.Event, stream=None) -> None:
    """Record `event` as a timestamp node (usable inside stream capture)."""
    rc = lib().slx_event_record_external(event.cuda_event, stream_ptr(stream))
    _check("slx_event_record_external", rc)


def event_elapsed_many(starts, ends) -> np.ndarray:
    """Elapsed ms of n (start, end) event pairs (both already completed)."""
    n = len(starts)
    a = (C.c_void_p * n)(*[e.cuda_event for e in starts])
    b = (C.c_void_p * n)(*[e.cuda_event for e in ends])
    out = (C.c_float * n)()
    rc = lib().slx_event_elapsed_many(a, b, n, out)
    _check("slx_event_elapsed_many", rc)
    return np.frombuffer(out, dtype=np.float32).copy()


def qk_norm_rope_cache(qkv, n_q, n_kv, hd, q_norm, k_norm, eps, inv_freq,
                       pos, k_cache, v_cache, status, stream=None) -> None:
    rc = lib().slx_qk_norm_rope_cache(
        qkv.data_ptr(), qkv.shape[0], n_q, n_kv, hd, q_norm.data_ptr(),
        k_norm.data_ptr(), eps, inv_freq.data_ptr(), pos.data_ptr(),
        k_cache.shape[0], k_cache.data_ptr(), v_cache.data_ptr(),
        status.data_ptr(), stream_ptr(stream))
    _check("slx_qk_norm_rope_cache", rc)
    _count(1)


def attn_decode(qkv, n_q, n_kv, hd, k_cache, v_cache, pos, out,
                stream=None) -> None:
    rc = lib().slx_attn_decode(qkv.data_ptr(), qkv.shape[0], n_q, n_kv, hd,
                               k_cache.data_ptr(), v_cache.data_ptr(),
                               pos.data_ptr(), k_cache.shape[0], out.data_ptr(),
                               stream_ptr(stream))
    _check("slx_attn_decode", rc)
    _count(1)


def attn_rope_decode(qkv, n_q, n_kv, hd, q_norm, k_norm, eps, inv_freq, pos,
                     k_cache, v_cache, out, status, stream=None) -> None:
    """One decode token: q/k norm + RoPE + cache append + attention."""
    rc = lib().slx_attn_rope_decode(
        qkv.data_ptr(), n_q, n_kv, hd, q_norm.data_ptr(), k_norm.data_ptr(),
        eps, inv_freq.data_ptr(), pos.data_ptr(), k_cache.shape[0],
        k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
        status.data_ptr(), stream_ptr(stream))
    _check("slx_attn_rope_decode", rc)
    _count(1)


def argmax(logits, out, stream=None) -> None:
    T, V = logits.shape[-2], logits.shape[-1]
    rc = lib().slx_argmax(logits.data_ptr(), T, V, out.data_ptr(),
                          stream_ptr(stream))
    _check("slx_argmax", rc)
    _count(1)


def pread_many(fds: np.ndarray, offsets: np.ndarray, sizes: np.ndarray,
               dsts: np.ndarray, threads: int) -> tuple[int, int, int]:
    """Native batched pread (host only).  Arrays: int32 fds, int64 offsets
    and sizes, uint64 destination addresses.  Returns (rc, failed index,
    errno of the failure, 0 = end of file)."""
    n = len(fds)
    fi, fe = C.c_int(-1), C.c_int(0)
    rc = lib().slx_pread_many(fds.ctypes.data, offsets.ctypes.data,
                              sizes.ctypes.data, dsts.ctypes.data, n, threads,
                              C.byref(fi), C.byref(fe))
    return int(rc), fi.value, fe.value


def copy_many(dsts: list[int], srcs: list[int], sizes: list[int],
              stream: torch.cuda.Stream | None = None) -> None:
    n = len(dsts)
    if n == 0:
        return
    D = (C.c_void_p * n)(*dsts)
    S = (C.c_void_p * n)(*srcs)
    Z = (C.c_size_t * n)(*sizes)
    rc = lib().slx_copy_many(D, S, Z, n, stream_ptr(stream))
    _check("slx_copy_many", rc)


def prefill_scratch_bytes(n_blocks: int, hidden: int, inter: int,
                          bits: int) -> int:
    return int(lib().slx_prefill_scratch_bytes(n_blocks, hidden, inter, bits))


def prefill_grouped(bank: slx_expert_bank, x: torch.Tensor,
                    pair_row: torch.Tensor, blocks: torch.Tensor,
                    out: torch.Tensor, scratch: torch.Tensor,
                    status: torch.Tensor, out_row: torch.Tensor | None = None,
                    stream: torch.cuda.Stream | None = None) -> None:
    """Expert-major prefill over pair blocks (int32 [n_blocks, 4] = slot,
    first pair, pairs, 0); out [n_out, H] per-pair unweighted outputs."""
    rc = lib().slx_prefill_grouped(
        C.byref(bank), x.data_ptr(), x.shape[0], pair_row.data_ptr(),
        pair_row.numel(), blocks.data_ptr(), blocks.shape[0], ptr(out_row),
        out.data_ptr(), out.shape[0], scratch.data_ptr(),
        scratch.numel() * scratch.element_size(), status.data_ptr(),
        stream_ptr(stream))
    _check("slx_prefill_grouped", rc)
    _count(3)
