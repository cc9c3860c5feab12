"""Operand-range edges of the expert kernels: either the tolerance holds or
the call is rejected with SLX_ERR_RANGE -- never a silent divergence.

The tensor-core prefill forms s*q, b and the activations in fp16; that is
exact for 2^-17 <= |s| < 64, 2^-17 <= |b| < 65504 (0 exact), activations and
group sums below 65504 (include/streamlx_cuda.h, slx_prefill.cu).  Outside
that the kernel reports SLX_ERR_RANGE and ops.prefill_grouped reruns the
call on the GEMV kernels (scales and biases in fp32); an activation the GEMV
kernels cannot hold either (|x| >= 65504 after the code-position factor, or
a SwiGLU output that large) is rejected with SLX_ERR_RANGE."""

import ml_dtypes
import numpy as np
import pytest
import torch

from oracle import affine as A

from .kernel_cases import bf16_np, bf16_tensor, check_close, make_bank, pack_pool

pytestmark = pytest.mark.gpu
E, H, I = 2, 512, 512


def _bits(v: float) -> int:
    return int(np.array([v], np.float32).astype(ml_dtypes.bfloat16)
               .view(np.uint16)[0])


def _bank(edit):
    """Bank of E 2-bit experts with `edit(tt, npt)` applied to both copies
    before packing (slot s = expert s)."""
    from streamlx_b200 import _lib as L
    tt, npt, qp = make_bank(E, H, I, 2, seed=21)
    tt = {p: tuple(t.cpu().clone() for t in v) for p, v in tt.items()}
    edit(tt, npt)
    pool, stride = pack_pool(tt, list(range(E)), H, I, 2)
    return L.bank_struct(pool, E, H, I, 2, stride), pool, npt, qp


def _set(tt, npt, proj, part, e, row, grp, value):
    b = _bits(value)
    idx = {"scales": 1, "biases": 2}[part]
    tt[proj][idx].view(torch.int16)[e, row, grp] = np.int16(np.uint16(b)
                                                             .view(np.int16))
    npt[proj][part][e, row, grp] = b


def _prefill(bank, x, experts):
    from streamlx_b200 import ops
    P = len(experts)
    pair_row = np.arange(P, dtype=np.int32) % x.shape[0]
    order = np.argsort(experts, kind="stable")
    slots, counts = np.unique(np.asarray(experts)[order], return_counts=True)
    out = ops.prefill_grouped(bank, bf16_tensor(x), pair_row[order], slots,
                              counts, out_row=order, n_out=P)
    torch.cuda.synchronize()
    return bf16_np(out), pair_row


def _want(npt, qp, x, pair_row, experts):
    w = np.zeros((len(experts), H), np.float32)
    for i, e in enumerate(experts):
        w[i] = A.expert_forward(x[pair_row[i]][None],
                                A.dequant_expert(npt, int(e), qp))[0]
    return w


EXPERTS = [0] * 40 + [1] * 30


@pytest.mark.parametrize("part,value,rerouted", [
    ("scales", 63.75, False),        # just below the fp16 bound: exact
    ("scales", 64.0, True),          # 1024 * s overflows fp16: rerouted
    ("scales", 2.0 ** -18, True),    # s*q loses bits in fp16: rerouted
    ("biases", 2.0 ** -16, False),   # fp16 subnormal, still exact
    ("biases", 2.0 ** -18, True),    # below the subnormal step: rerouted
])
def test_prefill_scale_bias_edges(part, value, rerouted):
    from streamlx_b200 import _lib as L

    def edit(tt, npt):
        for row in (3, 200):
            _set(tt, npt, "gate_proj", part, 0, row, 1, value)
            _set(tt, npt, "down_proj", part, 1, row, 2, value)
    bank, pool, npt, qp = _bank(edit)
    rng = np.random.default_rng(4)
    x = A.bf16_round(rng.standard_normal((24, H)).astype(np.float32) * 0.25)
    # the tensor-core kernel's own verdict on these operands
    from streamlx_b200 import ops
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    order = np.argsort(EXPERTS, kind="stable")
    slots, counts = np.unique(np.asarray(EXPERTS)[order], return_counts=True)
    blocks = torch.as_tensor(ops.prefill_blocks(slots, counts), device="cuda")
    pr = torch.as_tensor((np.arange(len(EXPERTS)) % 24)[order]
                         .astype(np.int32), device="cuda")
    out = torch.empty(len(EXPERTS), H, dtype=torch.bfloat16, device="cuda")
    sc = torch.empty(L.prefill_scratch_bytes(blocks.shape[0], H, I, 2),
                     dtype=torch.uint8, device="cuda")
    L.prefill_grouped(bank, bf16_tensor(x), pr, blocks, out, sc, st)
    torch.cuda.synchronize()
    assert int(st.item()) == (L.SLX_ERR_RANGE if rerouted else 0)
    got, pair_row = _prefill(bank, x, EXPERTS)       # rerouted when needed
    check_close(got, _want(npt, qp, x, pair_row, EXPERTS))


def test_prefill_small_and_moderate_activations_pass():
    """Activations of 1e-6 (fp16 subnormals, error < 2^-25 each) and
    outliers of 40 stay within the tolerance on the tensor-core path."""
    bank, pool, npt, qp = _bank(lambda tt, npt: None)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((24, H)).astype(np.float32)
    x[:, ::7] = 1e-6
    x[3, 17] = 40.0
    x = A.bf16_round(x)
    got, pair_row = _prefill(bank, x, EXPERTS)
    check_close(got, _want(npt, qp, x, pair_row, EXPERTS))


def test_outlier_activations_are_rejected():
    """3e4 outliers: the prefill's group sums leave fp16 (rerouted) and the
    SwiGLU outputs they drive leave it too -- the call is rejected with
    SLX_ERR_RANGE, not answered wrongly."""
    from streamlx_b200 import _lib as L
    bank, pool, npt, qp = _bank(lambda tt, npt: None)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((24, H)).astype(np.float32)
    x[2, 64:67] = 3e4
    x = A.bf16_round(x)
    with pytest.raises(L.SlxError) as ei:
        _prefill(bank, x, EXPERTS)
    assert ei.value.rc == L.SLX_ERR_RANGE


def test_decode_gemv_scale_edges_and_rejection():
    """The decode kernel keeps scales and biases in fp32: a scale of 96 is
    exact there; an activation of 7e4 cannot enter its fp16 fragments and
    is reported as SLX_ERR_RANGE."""
    from streamlx_b200 import _lib as L, ops

    def edit(tt, npt):
        _set(tt, npt, "gate_proj", "scales", 0, 5, 0, 96.0)
        _set(tt, npt, "up_proj", "biases", 1, 9, 3, 2.0 ** -20)
    bank, pool, npt, qp = _bank(edit)
    rng = np.random.default_rng(7)
    x = A.bf16_round(rng.standard_normal((1, H)).astype(np.float32) * 0.25)
    ids = torch.tensor([[0, 1]], dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = ops.switchglu(bank, bf16_tensor(x), ids, 2, inter=I, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    want = np.stack([A.expert_forward(x, A.dequant_expert(npt, e, qp))[0]
                     for e in (0, 1)])
    check_close(bf16_np(y)[0], want)
    x[0, 96] = 7e4          # a column whose code-position factor is 1
    x = A.bf16_round(x)
    ops.switchglu(bank, bf16_tensor(x), ids, 2, inter=I, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == L.SLX_ERR_RANGE
