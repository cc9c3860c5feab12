"""Expert-major prefill kernel (tcgen05) against the CPU oracle.

The reference's expert-major sweep (streamlx/integrate.py:141-232) runs
switch_forward (streamlx/pool.py:30-50) over the (token, expert) pairs of
each batch of experts; slx_prefill_grouped computes those per-pair outputs
for pairs grouped by expert.  Checked: per-pair outputs within the bf16
tolerance (max-abs 2e-2, rel-L2 1e-3) of the oracle's correctly rounded
bf16 pipeline, ragged and split blocks, scattered output rows, identical
bits on a repeated call, and a block that names a slot outside the pool
(skipped, SLX_ERR_OUT_OF_RANGE).
"""

import numpy as np
import pytest
import torch

from oracle import affine as A
from .kernel_cases import (bf16_np, bf16_tensor, check_close, make_bank,
                                pack_pool)

pytestmark = pytest.mark.gpu


def _case(E, H, I, counts, seed, n_tok=None):
    """Bank of E 2-bit experts packed into slots (slot s = expert E-1-s),
    token rows x, and pairs grouped by expert: counts[e] pairs of expert e."""
    from streamlx_b200 import _lib as L
    tt, npt, qp = make_bank(E, H, I, 2, seed)
    slot_of = {e: E - 1 - e for e in range(E)}
    pool, stride = pack_pool(tt, [E - 1 - s for s in range(E)], H, I, 2)
    bank = L.bank_struct(pool, E, H, I, 2, stride)
    rng = np.random.default_rng(seed)
    P = int(sum(counts))
    n_tok = n_tok or max(P // 2, 1)
    x = A.bf16_round(rng.standard_normal((n_tok, H)).astype(np.float32))
    pair_row = rng.integers(0, n_tok, P).astype(np.int32)
    experts = [e for e in range(E) for _ in range(counts[e])]
    return bank, pool, npt, qp, x, pair_row, experts, slot_of


def _oracle(npt, qp, x, pair_row, experts):
    want = np.zeros((len(experts), x.shape[1]), dtype=np.float32)
    experts = np.asarray(experts)
    for e in np.unique(experts):
        deq = A.dequant_expert(npt, int(e), qp)
        sel = np.nonzero(experts == e)[0]
        want[sel] = A.expert_forward(x[pair_row[sel]], deq)
    return want


@pytest.mark.parametrize("E,H,I,counts", [
    (3, 512, 512, [5, 16, 37]),                 # ragged, single blocks
    (4, 1024, 512, [1, 130, 0, 64]),            # a split block, an empty expert
    (3, 2560, 1024, [40, 129, 7]),              # the 117B-shaped layer
])
def test_prefill_matches_oracle(E, H, I, counts):
    from streamlx_b200 import ops
    bank, pool, npt, qp, x, pair_row, experts, slot_of = _case(
        E, H, I, counts, seed=7 + H + I)
    xt = bf16_tensor(x)
    slots = [slot_of[e] for e in range(E) if counts[e]]
    cnts = [c for c in counts if c]
    out = ops.prefill_grouped(bank, xt, pair_row, slots, cnts)
    torch.cuda.synchronize()
    ops.check_status(xt.device)
    got = bf16_np(out)
    want = _oracle(npt, qp, x, pair_row, experts)
    check_close(got, want)


def test_prefill_out_rows_and_repeat_agree():
    """Scattered output rows; a second call gives identical bits (every
    reduction runs in a fixed order)."""
    from streamlx_b200 import ops
    E, H, I, counts = 3, 512, 512, [20, 3, 50]
    bank, pool, npt, qp, x, pair_row, experts, slot_of = _case(E, H, I,
                                                               counts, seed=3)
    P = sum(counts)
    perm = np.random.default_rng(5).permutation(P).astype(np.int32)
    xt = bf16_tensor(x)
    slots = [slot_of[e] for e in range(E)]
    outs = [ops.prefill_grouped(bank, xt, pair_row, slots, counts,
                                out_row=perm, n_out=P) for _ in range(2)]
    torch.cuda.synchronize()
    ops.check_status(xt.device)
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    want = _oracle(npt, qp, x, pair_row, experts)
    got = bf16_np(outs[0])[perm]
    check_close(got, want)


def test_prefill_bad_block_is_skipped_with_status():
    from streamlx_b200 import _lib as L
    from streamlx_b200 import ops
    E, H, I, counts = 2, 512, 512, [8, 8]
    bank, pool, npt, qp, x, pair_row, experts, slot_of = _case(E, H, I,
                                                               counts, seed=11)
    xt = bf16_tensor(x)
    dev = xt.device
    blocks = torch.tensor([[slot_of[0], 0, 8, 0], [E + 5, 8, 8, 0]],
                          dtype=torch.int32, device=dev)
    pr = torch.as_tensor(pair_row, device=dev)
    out = torch.zeros(16, H, dtype=torch.bfloat16, device=dev)
    need = L.prefill_scratch_bytes(2, H, I, 2)
    sc = torch.empty(need, dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    L.prefill_grouped(bank, xt, pr, blocks, out, sc, st)
    torch.cuda.synchronize()
    assert int(st.item()) == -4          # SLX_ERR_OUT_OF_RANGE
    got = bf16_np(out)
    want = _oracle(npt, qp, x, pair_row[:8], experts[:8])
    check_close(got[:8], want)
    assert not got[8:].any()             # the bad block wrote nothing


@pytest.mark.parametrize("n_slots,mode", [(12, "sweep"), (64, "pool")])
def test_wrapper_prefill_on_tensor_cores(tmp_path, monkeypatch, n_slots, mode):
    """StreamingSwitchGLU on a 2-bit layer: a 48-token prefill whose expert
    union exceeds the pool runs the expert-major sweep, one that fits runs
    the in-pool grouped path; both go through slx_prefill_grouped and must
    equal the oracle's switch_forward (streamlx/pool.py:30-50)."""
    from oracle.model import OracleDecoder
    from streamlx_b200 import _lib as L
    from streamlx_b200 import synth
    from streamlx_b200.integrate import StreamingSwitchGLU
    from streamlx_b200.pool import StreamingSwitchMLP
    from streamlx_b200.reader import ExpertReader
    from streamlx_b200.stindex import SafetensorsIndex
    monkeypatch.setenv("STREAMLX_PREFILL", "sweep")
    cfg = synth.SynthConfig(name="pf2", hidden=512, layers=1, n_experts=64,
                            top_k=4, inter=512, expert_bits=2, zipf_s=1.1)
    d = synth.write_model(str(tmp_path / "pf2"), cfg, seed=5)
    index = SafetensorsIndex(d)
    pool = StreamingSwitchMLP(d, 0, n_slots, index=index,
                              reader=ExpertReader(index))
    w = StreamingSwitchGLU(pool)
    rng = np.random.default_rng(9)
    T = 48
    if mode == "pool":       # 16 distinct experts: fits the 64-slot pool
        cand = rng.choice(cfg.n_experts, 16, replace=False)
        ids = np.stack([rng.choice(cand, 4, replace=False) for _ in range(T)])
    else:
        ids = np.stack([rng.choice(cfg.n_experts, 4, replace=False)
                        for _ in range(T)])
    x = A.bf16_round(rng.standard_normal((T, cfg.hidden)).astype(np.float32))
    launches = L.LAUNCHES[0]
    y = w(bf16_tensor(x)[None], torch.as_tensor(ids[None].astype(np.int32)).cuda())
    torch.cuda.synchronize()
    assert L.LAUNCHES[0] > launches
    oracle = OracleDecoder(d)
    want = np.zeros((T, 4, cfg.hidden), dtype=np.float32)
    for e in np.unique(ids):
        sel = np.argwhere(ids == e)
        want[sel[:, 0], sel[:, 1]] = A.expert_forward(x[sel[:, 0]],
                                                      oracle.expert(0, int(e)))
    check_close(bf16_np(y)[0], want)
    if mode == "sweep":
        assert pool.sweep_experts > 0
    pool.reader.close()
