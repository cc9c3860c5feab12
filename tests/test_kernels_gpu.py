"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bars: dequantised weights and routing ids bit-exact; bf16 layer outputs
within max-abs 2e-2 and rel-L2 1e-3 (the tolerance written in
tests/kernel_cases.py).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle import tiles as OTI
from oracle import trunk as OT
from streamlx_b200 import _lib as L
from streamlx_b200 import synth

from .kernel_cases import (bf16_np, bf16_tensor, check_close, make_bank,
                           pack_pool, quant_stack, to_np)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    torch.cuda.init()
    return torch.device("cuda:0")


def _status(dev):
    return torch.zeros(1, dtype=torch.int32, device=dev)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_dequant_rows_bit_exact(dev, bits):
    E, out, inp = 3, 64, 512
    pk, s, b = quant_stack(E, out, inp, bits, seed=bits)
    w, sn, bn = to_np(pk, s, b)
    rows = torch.tensor([5, 0, 63, 17, 130, 191], dtype=torch.int32,
                        device=dev)
    o = torch.empty(len(rows), inp, dtype=torch.float32, device=dev)
    st = _status(dev)
    L.dequant_rows((pk.reshape(E * out, -1).to(dev),
                    s.reshape(E * out, -1).to(dev),
                    b.reshape(E * out, -1).to(dev)), inp, bits, rows,
                   len(rows), E * out, o, st)
    torch.cuda.synchronize()
    want = A.dequant(w.reshape(E * out, -1), sn.reshape(E * out, -1),
                     bn.reshape(E * out, -1), bits, 64)[rows.cpu().numpy()]
    got = o.cpu().numpy()
    assert st.item() == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("cfg", [(1024, 512, 4), (2560, 1024, 2),
                                 (512, 256, 8), (2048, 512, 4)])
def test_pack_experts_byte_exact(dev, cfg):
    H, I, bits = cfg
    tt, npt, _ = make_bank(3, H, I, bits, seed=H + bits, device="cpu")
    pool, stride = pack_pool(tt, [2, 0], H, I, bits)
    n = L.expert_tiled_bytes(H, I, bits)
    assert n == synth.expert_bytes(H, I, bits, 64)
    got = pool.cpu().numpy()
    for slot, e in enumerate([2, 0]):
        want = OTI.expert_tiled(*[(npt[p]["weight"][e], npt[p]["scales"][e],
                                   npt[p]["biases"][e])
                                  for p in ("gate_proj", "up_proj",
                                            "down_proj")], H, I, bits)
        assert got[slot * stride: slot * stride + n].tobytes() == want


@pytest.mark.parametrize("shape", [(272, 1024, 4), (96, 512, 2), (64, 256, 8)])
def test_pack_dense_byte_exact(dev, shape):
    out_f, in_f, bits = shape
    pk, s, b = quant_stack(1, out_f, in_f, bits, seed=3)
    w, sn, bn = to_np(pk[0], s[0], b[0])
    dst = torch.zeros(L.dense_tiled_bytes(out_f, in_f, bits), dtype=torch.uint8,
                      device=dev)
    L.pack_dense((pk[0].to(dev), s[0].to(dev), b[0].to(dev)), out_f, in_f,
                 bits, dst)
    torch.cuda.synchronize()
    assert dst.cpu().numpy().tobytes() == OTI.dense_tiled((w, sn, bn), out_f,
                                                          in_f, bits)


def _run_switchglu(dev, E, H, I, bits, k, T, n_slots, combined, seed,
                   shared_I=0):
    tt, npt, qp = make_bank(E, H, I, bits, seed, device="cpu")
    rng = np.random.default_rng(seed)
    # resident experts -> slots (random placement)
    resident = rng.choice(E, n_slots, replace=False)
    slots = rng.permutation(n_slots)
    table = np.full(E, -1, dtype=np.int32)
    table[resident] = slots
    inv = np.empty(n_slots, dtype=np.int64)
    inv[slots] = resident
    pool, stride = pack_pool(tt, inv.tolist(), H, I, bits)
    ids = np.stack([rng.choice(resident, k, replace=False) for _ in range(T)])
    x = rng.standard_normal((T, H)).astype(np.float32)
    x = A.bf16_round(x)
    sc = rng.random((T, k)).astype(np.float32)
    sc /= sc.sum(-1, keepdims=True)
    bank = L.bank_struct(pool, n_slots, H, I, bits, stride)
    shared = None
    sh_np = None
    if shared_I:
        st_, sn_, sq_ = make_bank(1, H, shared_I, bits, seed + 99, device="cpu")
        sh_pool, _ = pack_pool(st_, [0], H, shared_I, bits)
        shared = L.shared_struct(sh_pool, shared_I)
        sh_np = (sn_, sq_)
    xt = bf16_tensor(x, dev)
    idt = torch.from_numpy(ids.astype(np.int32)).to(dev)
    sct = torch.from_numpy(sc).to(dev)
    tab = torch.from_numpy(table).to(dev)
    out = torch.empty((T, H) if combined else (T, k, H), dtype=torch.bfloat16,
                      device=dev)
    scratch = torch.zeros(L.switchglu_scratch_bytes(T, k, I, shared_I),
                          dtype=torch.uint8, device=dev)
    st = _status(dev)
    L.switchglu(bank, xt, idt, out, scratch, st,
                scores=sct if combined else None, slot_table=tab,
                shared=shared)
    torch.cuda.synchronize()
    assert st.item() == 0
    y = A.switch_forward(x[None], ids[None], npt, qp)[0]   # [T,k,H]
    if combined:
        sh = None
        if shared_I:
            sn_, sq_ = sh_np
            deq = A.dequant_expert(sn_, 0, sq_)
            sh = np.stack([A.expert_forward(x[t][None], deq)[0]
                           for t in range(T)])
        want = A.moe_combine(y, sc, sh)
    else:
        want = y
    return bf16_np(out), want


@pytest.mark.parametrize("case", [
    # E, H, I, bits, k, T, n_slots, combined, shared_I
    (32, 1024, 512, 4, 4, 1, 8, False, 0),      # config-1 layer, drop-in mode
    (32, 1024, 512, 4, 4, 1, 8, True, 0),       # config-1, fused combine
    (64, 2560, 1024, 2, 10, 1, 16, True, 0),    # config-3 expert shapes
    (64, 2560, 1024, 2, 10, 1, 16, False, 0),
    (48, 2048, 512, 4, 8, 1, 16, True, 512),    # config-2 with shared expert
    (16, 512, 256, 8, 2, 3, 6, True, 0),        # 8-bit, 3 tokens
    (32, 1024, 512, 4, 4, 5, 12, True, 256),    # 5 tokens + shared
])
@pytest.mark.parametrize("fused", [True, False])
def test_switchglu_parity(dev, case, fused):
    """Decode calls (T == 1) run as one cooperative launch by default; the
    two-launch path serves every T."""
    E, H, I, bits, k, T, ns, comb, shI = case
    if fused and T != 1:
        pytest.skip("the single-launch path serves decode calls only")
    prev = L.set_switchglu_fused(fused)
    try:
        for seed in (7, 8):     # twice: the grid barrier words are reused
            got, want = _run_switchglu(dev, E, H, I, bits, k, T, ns, comb,
                                       seed=seed, shared_I=shI)
            check_close(got, want)
            if T == 1:
                assert L.lib().slx_switchglu_last_kernels() == \
                    (1 if fused else 2)
    finally:
        L.set_switchglu_fused(prev)


@pytest.mark.parametrize("fused", [True, False])
def test_switchglu_unmapped_expert_sets_status(dev, fused):
    prev = L.set_switchglu_fused(fused)
    try:
        _unmapped_case(dev)
    finally:
        L.set_switchglu_fused(prev)


def _unmapped_case(dev):
    E, H, I, bits, k, ns = 16, 512, 256, 4, 2, 4
    tt, _, _ = make_bank(E, H, I, bits, 3, device="cpu")
    pool, stride = pack_pool(tt, list(range(ns)), H, I, bits)
    bank = L.bank_struct(pool, ns, H, I, bits, stride)
    table = torch.full((E,), -1, dtype=torch.int32, device=dev)
    table[:ns] = torch.arange(ns, dtype=torch.int32, device=dev)
    ids = torch.tensor([[1, 9]], dtype=torch.int32, device=dev)  # 9 unmapped
    x = torch.randn(1, H, device=dev).to(torch.bfloat16)
    out = torch.empty(1, k, H, dtype=torch.bfloat16, device=dev)
    scratch = torch.zeros(L.switchglu_scratch_bytes(1, k, I), dtype=torch.uint8,
                          device=dev)
    st = _status(dev)
    L.switchglu(bank, x, ids, out, scratch, st, slot_table=table)
    torch.cuda.synchronize()
    assert st.item() == -5   # SLX_ERR_UNMAPPED_EXPERT
    assert torch.all(out[0, 1] == 0)


def test_switchglu_host_errors(dev):
    E, H, I, bits = 8, 512, 256, 4
    tt, _, _ = make_bank(E, H, I, bits, 3, device="cpu")
    pool, stride = pack_pool(tt, list(range(E)), H, I, bits)
    bank = L.bank_struct(pool, E, H, I, 3, stride)  # 3-bit: unsupported
    x = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
    ids = torch.zeros(1, 2, dtype=torch.int32, device=dev)
    out = torch.empty(1, 2, H, dtype=torch.bfloat16, device=dev)
    scratch = torch.empty(1 << 16, dtype=torch.uint8, device=dev)
    with pytest.raises(L.SlxError):
        L.switchglu(bank, x, ids, out, scratch, _status(dev))
    bank.bits = 4
    with pytest.raises(L.SlxError):   # scratch too small
        L.switchglu(bank, x, ids, out, scratch[:16], _status(dev))
    bank.slot_stride = 16            # stride smaller than one expert
    with pytest.raises(L.SlxError):
        L.switchglu(bank, x, ids, out, scratch, _status(dev))


@pytest.mark.parametrize("shape", [(4608, 2048, 4, 1), (1024, 512, 4, 2),
                                   (2560, 3072, 4, 1), (512, 2560, 2, 1),
                                   (272, 1024, 8, 1),
                                   (40960, 512, 4, 1)])   # two CTAs per SM
def test_qlinear_parity(dev, shape):
    out_f, in_f, bits, T = shape
    pk, s, b = quant_stack(1, out_f, in_f, bits, seed=out_f)
    w, sn, bn = to_np(pk[0], s[0], b[0])
    deq = A.dequant(w, sn, bn, bits, 64)
    rng = np.random.default_rng(1)
    x = A.bf16_round(rng.standard_normal((T, in_f)).astype(np.float32))
    y = torch.empty(T, out_f, dtype=torch.bfloat16, device=dev)
    st = _status(dev)
    wt = torch.zeros(L.dense_tiled_bytes(out_f, in_f, bits), dtype=torch.uint8,
                     device=dev)
    L.pack_dense((pk[0].to(dev), s[0].to(dev), b[0].to(dev)), out_f, in_f,
                 bits, wt)
    L.qlinear(wt, out_f, in_f, bits, bf16_tensor(x, dev), y, st)
    torch.cuda.synchronize()
    assert st.item() == 0
    check_close(bf16_np(y), A.qmv(x, deq))


@pytest.mark.parametrize("T", [6, 1])    # 1: the many-SM one-token form
@pytest.mark.parametrize("mode", ["plain", "ratio", "forced"])
def test_router_parity(dev, mode, T):
    H, E, k = 2560, 256, 10
    rng = np.random.default_rng(5)
    x = A.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    wg = A.bf16_round((rng.standard_normal((E, H)) / np.sqrt(H))
                      .astype(np.float32))
    bias = synth.zipf_bias(E, 1.1, 3)
    ratio = None
    xin = x
    if mode == "ratio":
        ratio = A.bf16_round((1 + 0.05 * rng.standard_normal(H))
                             .astype(np.float32))
        xin = A.bf16_round(x * ratio)
    force = forced = None
    if mode == "forced":
        force = np.array([1, 0, 1, 0, 0, 1][:T], dtype=np.int32)
        forced = np.stack([rng.choice(E, k, replace=False)
                           for _ in range(T)]).astype(np.int32)
    ids_w, sc_w, _ = A.router(xin, A.bf16_to_bits(wg), bias, k, True)
    if mode == "forced":
        f_ids, f_sc, _ = A.router(xin, A.bf16_to_bits(wg), bias, k, True,
                                  forced_ids=forced)
        m = force.astype(bool)
        ids_w[m], sc_w[m] = f_ids[m], f_sc[m]
    oi = torch.empty(T, k, dtype=torch.int32, device=dev)
    os_ = torch.empty(T, k, dtype=torch.float32, device=dev)
    scratch = torch.zeros(L.router_scratch_bytes(T, E), dtype=torch.uint8,
                          device=dev)
    st = _status(dev)
    for _ in range(2):   # tickets must be left at zero for the next call
        L.router_topk(bf16_tensor(x, dev), bf16_tensor(wg, dev),
                      torch.from_numpy(bias).to(dev), k, True, oi, os_,
                      scratch, st,
                      ratio=None if ratio is None else bf16_tensor(ratio, dev),
                      force=None if force is None else
                      torch.from_numpy(force).to(dev),
                      forced_ids=None if forced is None else
                      torch.from_numpy(forced).to(dev))
        torch.cuda.synchronize()
        assert st.item() == 0
        assert np.array_equal(oi.cpu().numpy(), ids_w)
        np.testing.assert_allclose(os_.cpu().numpy(), sc_w, rtol=1e-5,
                                   atol=1e-7)


def test_router_ties_lower_id(dev):
    T, H, E, k = 1, 64, 16, 4
    x = np.zeros((T, H), dtype=np.float32)
    wg = np.zeros((E, H), dtype=np.float32)
    bias = np.array([0, 1, 1, 0, 2, 1, 0, 2, 0, 0, 0, 0, 0, 0, 0, 0],
                    dtype=np.float32)
    oi = torch.empty(T, k, dtype=torch.int32, device=dev)
    os_ = torch.empty(T, k, dtype=torch.float32, device=dev)
    scratch = torch.zeros(L.router_scratch_bytes(T, E), dtype=torch.uint8,
                          device=dev)
    L.router_topk(bf16_tensor(x, dev), bf16_tensor(wg, dev),
                  torch.from_numpy(bias).to(dev), k, False, oi, os_, scratch,
                  _status(dev))
    torch.cuda.synchronize()
    assert oi.cpu().numpy().tolist() == [[4, 7, 1, 2]]


def test_trunk_kernels(dev):
    rng = np.random.default_rng(9)
    T, H, eps = 1, 2048, 1e-6
    h = A.bf16_round(rng.standard_normal((T, H)).astype(np.float32) * 3)
    d = A.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    w = A.bf16_round((1 + 0.05 * rng.standard_normal(H)).astype(np.float32))
    ht, dt = bf16_tensor(h, dev), bf16_tensor(d, dev)
    y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    L.add_rmsnorm(ht, dt, bf16_tensor(w, dev), eps, y)
    torch.cuda.synchronize()
    hw, yw = OT.add_rmsnorm(h, d, w, eps)
    assert np.array_equal(bf16_np(ht), hw)
    check_close(bf16_np(y), yw)

    nq, nkv, hd, maxlen = 16, 2, 128, 64
    theta = 1e6
    inv = OT.rope_inv_freq(hd, theta)
    kc = torch.zeros(maxlen, nkv, hd, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    kc_np = np.zeros((maxlen, nkv, hd), np.float32)
    vc_np = np.zeros_like(kc_np)
    qn = A.bf16_round((1 + 0.05 * rng.standard_normal(hd)).astype(np.float32))
    kn = A.bf16_round((1 + 0.05 * rng.standard_normal(hd)).astype(np.float32))
    st = _status(dev)
    for p in range(20):
        qkv = A.bf16_round(rng.standard_normal((1, (nq + 2 * nkv) * hd))
                           .astype(np.float32))
        qkv_t = bf16_tensor(qkv, dev)
        pos = torch.tensor([p], dtype=torch.int32, device=dev)
        L.qk_norm_rope_cache(qkv_t, nq, nkv, hd, bf16_tensor(qn, dev),
                             bf16_tensor(kn, dev), eps,
                             torch.from_numpy(inv).to(dev), pos, kc, vc, st)
        att = torch.empty(1, nq * hd, dtype=torch.bfloat16, device=dev)
        L.attn_decode(qkv_t, nq, nkv, hd, kc, vc, pos, att)
        torch.cuda.synchronize()
        q = qkv[0, :nq * hd].reshape(nq, hd)
        kk = qkv[0, nq * hd:(nq + nkv) * hd].reshape(nkv, hd)
        vv = qkv[0, (nq + nkv) * hd:].reshape(nkv, hd)
        qr = np.stack([OT.qk_norm_rope(q[i], qn, eps, p, inv)
                       for i in range(nq)])
        kc_np[p] = np.stack([OT.qk_norm_rope(kk[i], kn, eps, p, inv)
                             for i in range(nkv)])
        vc_np[p] = vv
        check_close(bf16_np(kc[p]), kc_np[p])
        want = OT.attn_decode(qr, kc_np, vc_np, p + 1, nq, nkv)
        check_close(bf16_np(att).reshape(nq, hd), want)
    assert st.item() == 0

    V = 151936
    lg = A.bf16_round(rng.standard_normal((2, V)).astype(np.float32))
    lg[1, 77] = lg[1, 99] = 50.0
    out = torch.empty(2, dtype=torch.int32, device=dev)
    L.argmax(bf16_tensor(lg, dev), out)
    torch.cuda.synchronize()
    assert out.cpu().tolist() == [OT.argmax_first(lg[0]), 77]


@pytest.mark.parametrize("nq,nkv", [(16, 2), (24, 4)])
def test_attn_rope_one_launch_equals_two(dev, nq, nkv):
    """slx_attn_rope_decode (q/k norm + RoPE + cache append + attention in
    one launch) against slx_qk_norm_rope_cache + slx_attn_decode: the same
    bits in the output and in both caches, over 70 positions (two chunks of
    the attention's 64-position split)."""
    rng = np.random.default_rng(11)
    hd, maxlen, eps = 128, 96, 1e-6
    inv = torch.from_numpy(OT.rope_inv_freq(hd, 1e6)).to(dev)
    qn = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(hd))
                                  .astype(np.float32)), dev)
    kn = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(hd))
                                  .astype(np.float32)), dev)
    caches = [(torch.zeros(maxlen, nkv, hd, dtype=torch.bfloat16, device=dev),
               torch.zeros(maxlen, nkv, hd, dtype=torch.bfloat16, device=dev))
              for _ in range(2)]
    st = _status(dev)
    for p in range(70):
        qkv = bf16_tensor(A.bf16_round(
            rng.standard_normal((1, (nq + 2 * nkv) * hd)).astype(np.float32)),
            dev)
        pos = torch.tensor([p], dtype=torch.int32, device=dev)
        a1 = torch.empty(1, nq * hd, dtype=torch.bfloat16, device=dev)
        a2 = torch.empty_like(a1)
        q2 = qkv.clone()
        L.qk_norm_rope_cache(q2, nq, nkv, hd, qn, kn, eps, inv, pos,
                             caches[0][0], caches[0][1], st)
        L.attn_decode(q2, nq, nkv, hd, caches[0][0], caches[0][1], pos, a1)
        L.attn_rope_decode(qkv, nq, nkv, hd, qn, kn, eps, inv, pos,
                           caches[1][0], caches[1][1], a2, st)
        torch.cuda.synchronize()
        assert torch.equal(a1.view(torch.int16), a2.view(torch.int16)), p
    assert st.item() == 0
    for c0, c1 in zip(*caches):
        assert torch.equal(c0.view(torch.int16), c1.view(torch.int16))


@pytest.mark.parametrize("pos", [511, 512, 575, 599, 1040])
def test_attn_rope_long_context_equals_two(dev, pos):
    """The fused decode attention at positions whose chunks outnumber the
    cluster's CTAs (the first chunk staged before the wait, later ones
    after it, the token's own row substituted in either): same bits as the
    two-launch form over a randomly filled cache."""
    rng = np.random.default_rng(pos)
    nq, nkv, hd, maxlen, eps = 24, 4, 128, 1100, 1e-6
    inv = torch.from_numpy(OT.rope_inv_freq(hd, 1e6)).to(dev)
    qn = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(hd))
                                  .astype(np.float32)), dev)
    kn = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(hd))
                                  .astype(np.float32)), dev)
    fill = bf16_tensor(A.bf16_round(
        rng.standard_normal((maxlen, nkv, hd)).astype(np.float32)), dev)
    caches = [(fill.clone(), fill.clone()) for _ in range(2)]
    qkv = bf16_tensor(A.bf16_round(
        rng.standard_normal((1, (nq + 2 * nkv) * hd)).astype(np.float32)), dev)
    p = torch.tensor([pos], dtype=torch.int32, device=dev)
    st = _status(dev)
    a1 = torch.empty(1, nq * hd, dtype=torch.bfloat16, device=dev)
    a2 = torch.empty_like(a1)
    q2 = qkv.clone()
    L.qk_norm_rope_cache(q2, nq, nkv, hd, qn, kn, eps, inv, p,
                         caches[0][0], caches[0][1], st)
    L.attn_decode(q2, nq, nkv, hd, caches[0][0], caches[0][1], p, a1)
    L.attn_rope_decode(qkv, nq, nkv, hd, qn, kn, eps, inv, p,
                       caches[1][0], caches[1][1], a2, st)
    torch.cuda.synchronize()
    assert st.item() == 0
    assert torch.equal(a1.view(torch.int16), a2.view(torch.int16))
    for c0, c1 in zip(*caches):
        assert torch.equal(c0.view(torch.int16), c1.view(torch.int16))


def test_router_with_norm_equals_norm_then_router(dev):
    """slx_router_topk_multi_norm (residual add + RMSNorm + two router heads
    in one launch) against slx_add_rmsnorm_out + slx_router_topk_multi: the
    same bits in h_out, x_out, the ids and the scores."""
    H, E, k = 2560, 256, 10
    rng = np.random.default_rng(13)
    h = bf16_tensor(A.bf16_round(rng.standard_normal((1, H)).astype(np.float32) * 4), dev)
    d = bf16_tensor(A.bf16_round(rng.standard_normal((1, H)).astype(np.float32)), dev)
    w = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(H)).astype(np.float32)), dev)
    ratio = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(H)).astype(np.float32)), dev)
    gates = [bf16_tensor(A.bf16_round((rng.standard_normal((E, H)) / np.sqrt(H))
                                      .astype(np.float32)), dev) for _ in range(2)]
    bias = torch.from_numpy(synth.zipf_bias(E, 1.1, 3)).to(dev)
    st = _status(dev)
    outs = []
    for fused in (False, True):
        ho = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        xo = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
        ids = [torch.empty(1, k, dtype=torch.int32, device=dev) for _ in range(2)]
        sc = [torch.empty(1, k, dtype=torch.float32, device=dev) for _ in range(2)]
        scr = [torch.zeros(L.router_scratch_bytes(1, E), dtype=torch.uint8,
                           device=dev) for _ in range(2)]
        heads = [L.router_head(gates[0], bias, ids[0], sc[0], scr[0]),
                 L.router_head(gates[1], bias, ids[1], sc[1], scr[1],
                               ratio=ratio)]
        for _ in range(2):   # tickets left at zero for the next call
            if fused:
                L.router_topk_multi_norm(heads, h, d, w, 1e-6, ho, xo, E, k,
                                         True, st)
            else:
                L.add_rmsnorm_out(h, d, w, 1e-6, ho, xo)
                L.router_topk_multi(xo, heads, E, k, True, st)
        torch.cuda.synchronize()
        assert st.item() == 0
        outs.append([t.clone() for t in (ho, xo, *ids, *sc)])
    for a, b in zip(*outs):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_router_two_heads_one_launch(dev):
    """Router + next-layer predictor in one launch equal two single calls."""
    T, H, E, k = 3, 2048, 256, 8
    rng = np.random.default_rng(11)
    x = bf16_tensor(A.bf16_round(rng.standard_normal((T, H))
                                 .astype(np.float32)), dev)
    ws = [bf16_tensor(A.bf16_round((rng.standard_normal((E, H)) / np.sqrt(H))
                                   .astype(np.float32)), dev) for _ in range(2)]
    bs = [torch.from_numpy(synth.zipf_bias(E, 1.0, s)).to(dev) for s in (1, 2)]
    ratio = bf16_tensor(A.bf16_round((1 + 0.05 * rng.standard_normal(H))
                                     .astype(np.float32)), dev)
    force = torch.tensor([0, 1, 0], dtype=torch.int32, device=dev)
    forced = torch.from_numpy(np.stack([rng.choice(E, k, replace=False)
                                        for _ in range(T)]).astype(np.int32)
                              ).to(dev)
    st = _status(dev)

    def outs():
        return (torch.empty(T, k, dtype=torch.int32, device=dev),
                torch.empty(T, k, dtype=torch.float32, device=dev),
                torch.zeros(L.router_scratch_bytes(T, E), dtype=torch.uint8,
                            device=dev))
    single = [outs(), outs()]
    L.router_topk(x, ws[0], bs[0], k, True, *single[0], st, force=force,
                  forced_ids=forced)
    L.router_topk(x, ws[1], bs[1], k, True, *single[1], st, ratio=ratio)
    multi = [outs(), outs()]
    for _ in range(2):      # tickets left at zero for the next call
        heads = [L.router_head(ws[0], bs[0], *multi[0], force=force,
                               forced_ids=forced),
                 L.router_head(ws[1], bs[1], *multi[1], ratio=ratio)]
        L.router_topk_multi(x, heads, E, k, True, st)
        torch.cuda.synchronize()
        assert st.item() == 0
        for a, b in zip(single, multi):
            assert torch.equal(a[0], b[0])
            assert torch.equal(a[1], b[1])


@pytest.mark.parametrize("nq,nkv", [(16, 2), (24, 4), (4, 2)])
def test_attn_decode_chunks(dev, nq, nkv):
    """Split-K attention over chunk boundaries (64 positions per chunk)."""
    hd, maxlen = 128, 300
    rng = np.random.default_rng(nq)
    kc_np = A.bf16_round(rng.standard_normal((maxlen, nkv, hd))
                         .astype(np.float32))
    vc_np = A.bf16_round(rng.standard_normal((maxlen, nkv, hd))
                         .astype(np.float32))
    kc, vc = bf16_tensor(kc_np, dev), bf16_tensor(vc_np, dev)
    for p in (0, 63, 64, 127, 130, 299):
        qkv = A.bf16_round(rng.standard_normal((1, (nq + 2 * nkv) * hd))
                           .astype(np.float32))
        att = torch.empty(1, nq * hd, dtype=torch.bfloat16, device=dev)
        pos = torch.tensor([p], dtype=torch.int32, device=dev)
        for _ in range(2):          # tickets left at zero for the next call
            L.attn_decode(bf16_tensor(qkv, dev), nq, nkv, hd, kc, vc, pos,
                          att)
        torch.cuda.synchronize()
        want = OT.attn_decode(qkv[0, :nq * hd].reshape(nq, hd), kc_np, vc_np,
                              p + 1, nq, nkv)
        check_close(bf16_np(att).reshape(nq, hd), want)
