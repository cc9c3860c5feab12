"""Kernel-calling helpers around the pools (device side of the wrapper)."""

from __future__ import annotations

import torch

from . import _lib as L

_scratch: dict = {}

# When a list, every switchglu launch pair appends (start, end) CUDA events
# recorded around it on the current stream (the bench's roofline timing).
TIMING: list | None = None


def _status(device) -> torch.Tensor:
    key = ("status", device)
    t = _scratch.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _scratch[key] = t
    return t


def scratch(nbytes: int, device, tag: str = "glu") -> torch.Tensor:
    """Grow-only device scratch shared by calls on one device."""
    key = (tag, device)
    t = _scratch.get(key)
    if t is None or t.numel() < nbytes:
        # zeroed: the switchglu scratch ends with grid-barrier words
        t = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _scratch[key] = t
    return t


def check_status(device) -> None:
    """Raise if a kernel recorded a device-side error (synchronises)."""
    st = _status(device)
    v = int(st.item())
    if v != 0:
        st.zero_()
        raise L.SlxError("device", v, "device-side error status")


def as_bf16_2d(x: torch.Tensor) -> torch.Tensor:
    x = x.reshape(-1, x.shape[-1])
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    return x.contiguous()


def as_ids_2d(ids, k: int, device) -> torch.Tensor:
    if not isinstance(ids, torch.Tensor):
        ids = torch.as_tensor(ids)
    ids = ids.reshape(-1, k)
    if ids.dtype != torch.int32 or ids.device != device:
        ids = ids.to(device=device, dtype=torch.int32)
    return ids.contiguous()


def switchglu(bank, x2d: torch.Tensor, ids2d: torch.Tensor, k: int, *,
              scores: torch.Tensor | None = None, table: torch.Tensor | None = None,
              shared=None, out: torch.Tensor | None = None,
              inter: int, shared_inter: int = 0,
              scratch_buf: torch.Tensor | None = None,
              status: torch.Tensor | None = None) -> torch.Tensor:
    """One fused SwitchGLU launch pair.  scores None -> [T, k, H] per-expert
    unweighted outputs; else [T, H] combined (+ shared expert).
    ``scratch_buf`` / ``status`` override the per-device shared ones (a
    captured graph needs buffers that never move)."""
    T, H = x2d.shape
    dev = x2d.device
    if out is None:
        shape = (T, H) if scores is not None else (T, k, H)
        out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    sI = shared_inter if (scores is not None and shared is not None) else 0
    need = L.switchglu_scratch_bytes(T, k, inter, sI)
    if scratch_buf is not None:
        if scratch_buf.numel() * scratch_buf.element_size() < need:
            raise ValueError("switchglu: scratch_buf too small")
        sc = scratch_buf
    else:
        sc = scratch(need, dev)
    ev = None
    if TIMING is not None:
        ev = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
        ev[0].record()
    L.switchglu(bank, x2d, ids2d, out, sc,
                _status(dev) if status is None else status, scores=scores,
                slot_table=table, shared=shared if sI else None)
    if ev is not None:
        ev[1].record()
        TIMING.append((ev[0], ev[1], T, k, inter, sI))
    return out


def switch_forward_ids(pool, x, expert_ids) -> torch.Tensor:
    """streamlx/pool.py:299-304 on the pool: per-expert outputs [1,1,k,H]."""
    k = len(expert_ids)
    x2d = as_bf16_2d(x)
    pool.sync_device()
    ids = as_ids_2d(list(expert_ids), k, x2d.device)
    y = switchglu(pool.store.bank, x2d, ids, k, table=pool.store.table_dev,
                  inter=pool.inter)
    return y.reshape(1, 1, k, -1)


PREFILL_BLOCK = 128   # pairs per block (the kernel's MMA N)
# pairs per call from which the pool path uses the grouped tensor-core
# prefill instead of the per-token GEMV kernels
PREFILL_MIN_PAIRS = 64


def prefill_supported(hidden: int, inter: int, bits: int) -> bool:
    return bits == 2 and hidden % 512 == 0 and inter % 512 == 0 and \
        hidden <= 4096 and inter <= 4096


def prefill_blocks(slots, counts) -> "np.ndarray":
    """Blocks {slot, first pair, pairs, 0} of pairs grouped by expert:
    segment i (``counts[i]`` consecutive pairs of slot ``slots[i]``) is split
    into runs of at most PREFILL_BLOCK pairs."""
    import numpy as np
    rows = []
    p = 0
    for s, n in zip(slots, counts):
        n = int(n)
        for o in range(0, n, PREFILL_BLOCK):
            rows.append((int(s), p + o, min(PREFILL_BLOCK, n - o), 0))
        p += n
    return np.asarray(rows, dtype=np.int32).reshape(-1, 4)


def prefill_grouped(bank, x2d: torch.Tensor, pair_row, slots, counts, *,
                    out: torch.Tensor | None = None, out_row=None,
                    n_out: int | None = None) -> torch.Tensor:
    """Expert-major prefill on the tensor cores: pairs grouped by expert
    (``pair_row[p]`` = x row of pair p; segment i = ``counts[i]`` pairs of
    slot ``slots[i]``).  Returns per-pair unweighted outputs [P, H] (rows
    ``out_row[p]`` when given)."""
    import numpy as np
    dev = x2d.device
    H = x2d.shape[1]
    blocks = prefill_blocks(slots, counts)
    P = int(np.sum(counts)) if len(counts) else 0
    if out is None:
        out = torch.empty(n_out if n_out is not None else P, H,
                          dtype=torch.bfloat16, device=dev)
    if blocks.shape[0] == 0:
        return out
    pr = torch.as_tensor(np.asarray(pair_row, dtype=np.int32), device=dev)
    bl = torch.as_tensor(blocks, device=dev)
    orow = None if out_row is None else torch.as_tensor(
        np.asarray(out_row, dtype=np.int32), device=dev)
    need = L.prefill_scratch_bytes(blocks.shape[0], H, bank.inter, bank.bits)
    if need == 0:
        raise L.SlxError("slx_prefill_scratch_bytes", -2, "unsupported shape")
    sc = scratch(need, dev, tag="prefill")
    st = _status_word(dev, "prefill")
    L.prefill_grouped(bank, x2d, pr, bl, out, sc, st, out_row=orow)
    code = int(st.item())           # one sync per prefill call
    if code == 0:
        return out
    st.zero_()
    if code != L.SLX_ERR_RANGE:
        raise L.SlxError("slx_prefill_grouped", code, "device-side error")
    # an operand outside the tensor-core kernel's exact fp16 range: the
    # call runs on the GEMV kernels instead (fp32 scale/bias arithmetic)
    seg = np.repeat(np.asarray(slots, dtype=np.int32),
                    np.asarray(counts, dtype=np.int64))
    rows = torch.as_tensor(np.asarray(pair_row, dtype=np.int64), device=dev)
    xs = x2d[rows].contiguous()
    sid = torch.as_tensor(seg, device=dev).reshape(-1, 1)
    y = switchglu(bank, xs, sid, 1, inter=bank.inter,
                  status=st).reshape(-1, H)
    code = int(st.item())
    if code != 0:
        st.zero_()
        raise L.SlxError("prefill (GEMV path)", code,
                         "an activation is outside the fp16 range (|x| >= "
                         "65504) of the expert kernels")
    dst = torch.as_tensor(np.asarray(out_row if out_row is not None
                                     else np.arange(P), dtype=np.int64),
                          device=dev)
    out[dst] = y
    return out


def _status_word(device, tag: str) -> torch.Tensor:
    key = ("status", tag, device)
    t = _scratch.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _scratch[key] = t
    return t
