"""The V3 trunk's kernels (csrc/trunk.cu through the C ABI) against float64 restatements and against the CPU oracle
of the whole trunk (oracle/trunk.py, pinned to the reference's own decide_many logits by tests/golden/e2e_config1.npz).

Tolerances: od_gemm_f32 (3xTF32 on the tensor cores) within 5e-6 of sum_k |x_k w_k| per output element (fp32
accumulation of ~2^-21-accurate products); the split operand pairs within 2e-7 relative of their float64 value;
attention within 2e-6 of the float64 result on unit-normal q / k / v (5e-6 over 255-option rows: the fp32 q . k
over 64 dimensions is accurate to ~1e-6 of |q||k|); the whole trunk's logits within 5e-4 of the oracle's (fp32 summation
order differences through 4 layers)."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from opendecider_b200 import _lib
from opendecider_b200.v3 import TrunkConfig, V3Trunk, trunk_state_dict
from oracle import trunk as ot

pytestmark = pytest.mark.gpu


def _pair(x, cuda):
    return _lib.split_tf32(x.to(cuda).contiguous())


def _val(pair):
    return pair[0].double().cpu() + pair[1].double().cpu()


@pytest.mark.parametrize("M,N,K", [(1, 512, 4096), (300, 1368, 512), (257, 512, 1368), (1000, 1, 512),
                                   (129, 2736, 64), (64, 168, 64), (5000, 1536, 512)])
def test_gemm_f32_matches_fp64(cuda, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) / math.sqrt(K)
    b = torch.randn(N, generator=g)
    y = _lib.gemm_f32(_pair(x, cuda), _pair(w, cuda), bias=b.to(cuda)).cpu().double()
    ref = x.double() @ w.double().T + b.double()
    bound = x.double().abs() @ w.double().abs().T + b.double().abs()
    err = ((y - ref).abs() / bound).max().item()
    assert err < 5e-6, err


def test_gemm_f32_residual_scatter_and_broadcast(cuda):
    g = torch.Generator().manual_seed(1)
    M, N, K, R = 200, 512, 256, 500
    x, w, b = torch.randn(M, K, generator=g), torch.randn(N, K, generator=g) / 16, torch.randn(N, generator=g)
    rows = torch.randperm(R, generator=g)[:M]
    out = torch.randn(R, N, generator=g)
    exp = out.double().clone()
    exp[rows] += x.double() @ w.double().T + b.double()
    od = out.to(cuda)
    _lib.gemm_f32(_pair(x, cuda), _pair(w, cuda), bias=b.to(cuda), res=od, out=od, out_rows=rows.to(cuda))
    assert (od.cpu().double() - exp).abs().max().item() < 1e-4
    r1 = torch.randn(N, generator=g)                 # one residual row for every output row
    y = _lib.gemm_f32(_pair(x, cuda), _pair(w, cuda), res=r1.to(cuda)).cpu().double()
    assert (y - (r1.double() + x.double() @ w.double().T)).abs().max().item() < 1e-4


@pytest.mark.parametrize("dtype,n_mix,K", [(torch.bfloat16, 4, 4096), (torch.bfloat16, 3, 256), (torch.float32, 1, 512),
                                           (torch.float32, 1, 64), (torch.float32, 1, 1368)])
def test_scalenorm_split(cuda, dtype, n_mix, K):
    g = torch.Generator().manual_seed(K + n_mix)
    M = 77
    x = (torch.randn(M, n_mix * K, generator=g) * 3).to(dtype)
    gain = torch.tensor(math.sqrt(K) * 1.3)
    mw = torch.softmax(torch.randn(n_mix, generator=g), 0) if n_mix > 1 else None
    hi, lo = _lib.scalenorm_split(x.to(cuda), gain.to(cuda), mix_w=None if mw is None else mw.to(cuda))
    xd = x.double()
    v = (xd.view(M, n_mix, K) * mw.double()[None, :, None]).sum(1) if mw is not None else xd
    ref = gain.double() * v / v.norm(dim=-1, keepdim=True).clamp_min(1e-5)
    got = _val((hi, lo))
    assert ((got - ref).abs().max() / ref.abs().max()).item() < 2e-7
    hb = hi.cpu().view(torch.int32)
    assert int((hb & 0x1FFF).abs().max()) == 0                      # hi is a tf32 value
    assert bool((lo.cpu().abs() <= hi.cpu().abs() * 2.0 ** -11).all())   # lo: at most half a tf32 ulp of hi


def test_xatglu_split(cuda):
    g = torch.Generator().manual_seed(3)
    M, Fh = 300, 1368
    zv = torch.randn(M, 2 * Fh, generator=g) * 2
    a = torch.tensor(0.07)
    hi, lo = _lib.xatglu_split(zv.to(cuda), a.to(cuda))
    z, val = zv[:, :Fh].double(), zv[:, Fh:].double()
    ref = ((torch.atan(z) + math.pi / 2) / math.pi * (1 + 2 * a.double()) - a.double()) * val
    assert (_val((hi, lo)) - ref).abs().max().item() < 2e-6


def test_gemm_f32_rope_epilogue(cuda):
    """The RoPE the GEMM applies to the q / k columns as it writes them, against the oracle's rotation (v3.py:70-79)
    of the float64 product."""
    g = torch.Generator().manual_seed(9)
    M, K, H, Dh = 300, 512, 8, 64
    D = H * Dh
    x, w = torch.randn(M, K, generator=g), torch.randn(3 * D, K, generator=g) / math.sqrt(K)
    pos = torch.randint(0, 17000, (M,), generator=g)
    y = _lib.gemm_f32(_pair(x, cuda), _pair(w, cuda), rope_pos=pos.int().to(cuda), rope_inv=_lib.rope_table(Dh, cuda),
                      rope_cols=2 * D).cpu().double()
    ref = x.double() @ w.double().T
    rot = ot._rope_pairs(ref[:, :2 * D].view(1, M, 2 * H, Dh).transpose(1, 2), pos.view(1, M))
    ref[:, :2 * D] = rot.transpose(1, 2).reshape(M, 2 * D)
    bound = x.double().abs() @ w.double().abs().T
    pb = bound[:, :2 * D].view(M, D, 2).amax(-1, keepdim=True).expand(M, D, 2).reshape(M, 2 * D)
    bound[:, :2 * D] = pb                          # a rotated value mixes the two columns of its pair
    assert ((y - ref).abs() / bound).max().item() < 5e-6


def _attn_ref(q, k, v, bias):
    """float64 SDPA of (B, H, L, Dh) tensors with an additive mask, as the oracle's MHA calls it."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=bias)


@pytest.mark.parametrize("lens", [False, True])
@pytest.mark.parametrize("mode", ["self", "keys", "cls"])
@pytest.mark.parametrize("H,Dh", [(8, 64), (4, 16)])
def test_trunk_attn_modes(cuda, mode, H, Dh, lens):
    g = torch.Generator().manual_seed(H * 3 + len(mode))
    B, P, Tc, Kopt = 5, 70, 23, 9
    D = H * Dh
    # option ids: each question's options laid out contiguously, then padding (-1)
    gid = torch.full((B, P), -1, dtype=torch.long)
    pos = torch.zeros(B, P, dtype=torch.long)
    n_opt = [3, 9, 1, 6, 4]
    olen = torch.zeros(B, dtype=torch.long)
    for b in range(B):
        c = 0
        for k in range(n_opt[b]):
            n = int(torch.randint(1, 8, (1,), generator=g))
            gid[b, c:c + n] = k
            pos[b, c:c + n] = torch.arange(n)
            c += n
        olen[b] = c
    x_pad = gid < 0
    qlen = torch.tensor([23, 5, 17, 1, 12])
    c_pad = torch.arange(Tc)[None, :] >= qlen[:, None]
    cpos = torch.arange(Tc)[None, :] + torch.tensor([100, 7, 0, 2048, 33])[:, None]
    bonus = torch.randn(H, generator=g)
    if mode == "self":
        Lq, Lk = P, P
        q = torch.randn(B, Lq, D, generator=g)
        same = ((gid[:, :, None] == gid[:, None, :]) & ~x_pad[:, :, None]).double()
        bias = (bonus.double().view(1, H, 1, 1) * same[:, None]).masked_fill(x_pad[:, None, None, :], ot.NEG)
        qp, kp, kg, qg = pos, pos, gid, gid
        ql, kl = olen, olen
    elif mode == "keys":
        Lq, Lk = P, Tc
        q = torch.randn(B, Lq, D, generator=g)
        bias = torch.zeros(B, 1, 1, Tc, dtype=torch.float64).masked_fill(c_pad[:, None, None, :], ot.NEG)
        qp, kp, kg, qg = None, cpos, torch.where(c_pad, -1, 0), None
        ql, kl = olen, qlen
    else:
        Lq, Lk = Kopt, P
        q = torch.randn(1, 1, D, generator=g).expand(B, Lq, D)
        own = gid[:, None, :] == torch.arange(Kopt)[None, :, None]
        bias = torch.zeros(B, 1, Kopt, P, dtype=torch.float64).masked_fill(~own[:, None], ot.NEG)
        qp, kp, kg, qg = None, pos, gid, None
        ql, kl = torch.tensor(n_opt), olen
    if not lens:
        ql = kl = None
    k = torch.randn(B, Lk, D, generator=g)
    v = torch.randn(B, Lk, D, generator=g)
    # q and k arrive RoPE'd (the GEMM's epilogue): rotate them here in fp32 as the oracle does
    rot = lambda t, L, p: ot._rope_pairs(t.reshape(B, L, H, Dh).transpose(1, 2), p).transpose(1, 2).reshape(B, L, D)  # noqa: E731,E501
    q, k = rot(q, Lq, qp).contiguous(), rot(k, Lk, kp).contiguous()
    heads = lambda t, L: t.double().reshape(B, L, H, Dh).transpose(1, 2)   # noqa: E731
    ref = _attn_ref(heads(q, Lq), heads(k, Lk), heads(v, Lk), bias).transpose(1, 2).reshape(B * Lq, D)
    i32 = lambda t: None if t is None else t.int().contiguous().to(cuda)   # noqa: E731
    mcode = {"self": _lib.OD_TRUNK_SELF, "keys": _lib.OD_TRUNK_KEYS, "cls": _lib.OD_TRUNK_CLS}[mode]
    qd = q[0, :1].contiguous().to(cuda) if mode == "cls" else q.reshape(B * Lq, D).to(cuda)
    kv = torch.cat([k, v], -1).reshape(B * Lk, 2 * D).to(cuda)          # k | v side by side, as the GEMM writes
    kw = dict(k_grp=i32(kg), q_grp=i32(qg), bonus=bonus.to(cuda) if mode == "self" else None,
              q_shared=mode == "cls", q_len=i32(ql), k_len=i32(kl))
    o = _lib.trunk_attn(qd, kv[:, :D], kv[:, D:], mcode, B, Lq, Lk, H, pair=False, **kw).cpu().double()
    valid = torch.ones(B * Lq, dtype=torch.bool)
    if mode == "cls":   # options past a question's count see no key: zeros here (their logits are masked)
        valid = (torch.arange(Kopt)[None, :] < torch.tensor(n_opt)[:, None]).reshape(-1)
    if ql is not None:  # padding queries past q_len: zeros
        valid &= (torch.arange(Lq)[None, :] < ql[:, None]).reshape(-1)
    if not bool(valid.all()):
        assert o[~valid].abs().max().item() == 0.0
    assert (o[valid] - ref[valid]).abs().max().item() < 2e-6
    hi, lo = _lib.trunk_attn(qd, kv[:, :D], kv[:, D:], mcode, B, Lq, Lk, H, **kw)
    assert (_val((hi, lo)) - o).abs().max().item() < 1e-12


def _trunk_case(tc, n_q, seed):
    g = torch.Generator().manual_seed(seed)
    n_opt = torch.randint(2, 12, (n_q,), generator=g)
    o_lens = torch.randint(1, 6, (int(n_opt.sum()),), generator=g)
    q_lens = torch.randint(3, 40, (n_q,), generator=g)
    state_lens = torch.randint(10, 3000, (n_q,), generator=g)
    nf = tc.n_feat_layers * tc.d_feat
    q_flat = (torch.randn(int(q_lens.sum()), nf, generator=g) * 2).bfloat16()
    o_flat = (torch.randn(int(o_lens.sum()), nf, generator=g) * 2).bfloat16()
    lp = -torch.rand(int(o_lens.sum()), generator=g) * 5
    return q_lens, o_lens, n_opt, state_lens, q_flat, o_flat, lp


@pytest.mark.parametrize("size,lm", [("config1", False), ("config1", True), ("9b", False)])
def test_trunk_matches_oracle(cuda, size, lm):
    if size == "config1":
        tc = TrunkConfig(d_feat=256, n_feat_layers=3, d_model=64, n_heads=4, decision_layers=2, lm_feature=lm)
        n_q = 12
    else:
        tc = TrunkConfig(d_feat=4096, n_feat_layers=4, d_model=512, n_heads=8, decision_layers=4, lm_feature=lm)
        n_q = 24
    sd = trunk_state_dict(tc, seed=5)
    q_lens, o_lens, n_opt, sl, q_flat, o_flat, lp = _trunk_case(tc, n_q, seed=11)
    oracle = ot.OracleTrunk(tc, sd)
    ref = oracle.run(oracle.prepare(q_lens, o_lens, n_opt, sl), q_flat, o_flat, lp if lm else None)
    gpu = V3Trunk(tc, sd, cuda)
    got = gpu.run(gpu.prepare(q_lens, o_lens, n_opt, sl), q_flat.to(cuda), o_flat.to(cuda),
                  lp.to(cuda) if lm else None).cpu()
    mask = ref > ot.NEG / 2
    assert bool((got[~mask] == ot.NEG).all())
    d = (got[mask].double() - ref[mask].double()).abs().max().item()
    assert d < 5e-4, d
    assert np.isfinite(got.numpy()).all()


@pytest.mark.parametrize("mode", ["self", "cls"])
def test_trunk_attn_long_option_lists(cuda, mode):
    """Many key tiles (P = 700 option-token slots: eleven 64-key tiles through the cp.async double buffer) and many
    query blocks, against the float64 SDPA with the oracle's mask; 2 questions, 8 heads of 64."""
    g = torch.Generator().manual_seed(7)
    B, H, Dh, Kopt = 2, 8, 64, 255
    D = H * Dh
    lens = torch.randint(1, 4, (B, Kopt), generator=g)
    P = int(lens.sum(1).max())
    gid = torch.full((B, P), -1, dtype=torch.long)
    for b in range(B):
        gid[b, : int(lens[b].sum())] = torch.repeat_interleave(torch.arange(Kopt), lens[b])
    x_pad = gid < 0
    olen = (~x_pad).sum(1)
    bonus = torch.randn(H, generator=g)
    k = torch.randn(B, P, D, generator=g)
    v = torch.randn(B, P, D, generator=g)
    if mode == "self":
        Lq = P
        q = torch.randn(B, P, D, generator=g)
        same = ((gid[:, :, None] == gid[:, None, :]) & ~x_pad[:, :, None]).double()
        bias = (bonus.double().view(1, H, 1, 1) * same[:, None]).masked_fill(x_pad[:, None, None, :], ot.NEG)
        qd, kw = q.reshape(B * P, D), dict(q_grp=gid.int().to(cuda), bonus=bonus.to(cuda), q_len=olen.int().to(cuda))
        mcode = _lib.OD_TRUNK_SELF
    else:
        Lq = Kopt
        q = torch.randn(1, 1, D, generator=g).expand(B, Lq, D)
        own = gid[:, None, :] == torch.arange(Kopt)[None, :, None]
        bias = torch.zeros(B, 1, Kopt, P, dtype=torch.float64).masked_fill(~own[:, None], ot.NEG)
        qd, kw = q[0, :1].contiguous(), dict(q_shared=True, q_len=torch.full((B,), Kopt, dtype=torch.int32).to(cuda))
        mcode = _lib.OD_TRUNK_CLS
    heads = lambda t, L: t.double().reshape(B, L, H, Dh).transpose(1, 2)   # noqa: E731
    ref = _attn_ref(heads(q, Lq), heads(k, P), heads(v, P), bias).transpose(1, 2).reshape(B * Lq, D)
    kv = torch.cat([k, v], -1).reshape(B * P, 2 * D).to(cuda)
    o = _lib.trunk_attn(qd.to(cuda), kv[:, :D], kv[:, D:], mcode, B, Lq, P, H, k_grp=gid.int().to(cuda),
                        k_len=olen.int().to(cuda), pair=False, **kw).cpu().double()
    valid = torch.ones(B * Lq, dtype=torch.bool)
    if mode == "self":
        valid = (torch.arange(P)[None, :] < olen[:, None]).reshape(-1)
    assert (o[valid] - ref[valid]).abs().max().item() < 5e-6


def test_trunk_matches_oracle_255_options(cuda):
    """The whole trunk on config 5's question shape - 255 options of 1-3 tokens per question (P up to 765) - against
    the CPU oracle; 3 questions, the 9B trunk (d_model 512, 8 heads, 4 layers, 4 feature layers of 4096)."""
    tc = TrunkConfig(d_feat=4096, n_feat_layers=4, d_model=512, n_heads=8, decision_layers=4)
    sd = trunk_state_dict(tc, seed=6)
    g = torch.Generator().manual_seed(13)
    n_q = 3
    n_opt = torch.full((n_q,), 255)
    o_lens = torch.randint(1, 4, (int(n_opt.sum()),), generator=g)
    q_lens = torch.randint(20, 60, (n_q,), generator=g)
    sl = torch.tensor([16896, 16000, 900])
    nf = tc.n_feat_layers * tc.d_feat
    q_flat = (torch.randn(int(q_lens.sum()), nf, generator=g) * 2).bfloat16()
    o_flat = (torch.randn(int(o_lens.sum()), nf, generator=g) * 2).bfloat16()
    oracle = ot.OracleTrunk(tc, sd)
    ref = oracle.run(oracle.prepare(q_lens, o_lens, n_opt, sl), q_flat, o_flat)
    gpu = V3Trunk(tc, sd, cuda)
    got = gpu.run(gpu.prepare(q_lens, o_lens, n_opt, sl), q_flat.to(cuda), o_flat.to(cuda)).cpu()
    d = (got.double() - ref.double()).abs().max().item()
    assert d < 5e-4, d
