"""Parity of every libod_b200 kernel (called through the C ABI) with the CPU oracle and the reference's golden
outputs. Bytes, scales and int32 accumulators must match bit-exactly; floating-point outputs within the tolerance
written at each assert."""
import numpy as np
import pytest
import torch

from oracle import ops
from opendecider_b200 import _lib
from opendecider_b200 import synthetic as syn
from tests.conftest import from_bits

pytestmark = pytest.mark.gpu


def bf(a) -> torch.Tensor:
    return torch.as_tensor(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


# ------------------------------------------------------------------------------------------------ quantisers
def test_quant_rows_golden(cuda, golden):
    gc = syn.gemm_case(M=64, N=256, K=512, seed=1)
    for name, x, tdt in (("bf16", gc.x, torch.bfloat16), ("f16", gc.x.float().to(torch.float16), torch.float16),
                         ("f32", gc.x.float(), torch.float32)):
        q, s = _lib.quant_rows(x.to(cuda))
        assert np.array_equal(q.cpu().numpy(), golden[f"quant.{name}.q"]), name
        gs = golden[f"quant.{name}.scale"]
        gs = torch.from_numpy(gs) if tdt == torch.float32 else from_bits(gs, tdt)
        assert torch.equal(s.cpu().view(-1), gs.view(-1)), name
    q, s = _lib.quant_rows(gc.w.to(cuda))                      # A1: the weight quantiser
    assert np.array_equal(q.cpu().numpy(), golden["gemm.qweight"])
    assert torch.equal(s.cpu().view(-1), from_bits(golden["gemm.wscale"], torch.bfloat16).view(-1))


@pytest.mark.parametrize("M,K", [(1, 8), (7, 64), (513, 4096), (300, 12288), (2, 16384)])
def test_quant_rows_shapes(cuda, M, K):
    g = syn.gen(M * 7 + K)
    x = (torch.randn(M, K, generator=g) * torch.rand(M, 1, generator=g) * 10).to(torch.bfloat16)
    x[0, : min(K, 5)] = 0
    if M > 2:
        x[1] = 0                                                 # all-zero row: scale = 1e-8 / 127
    q, s = _lib.quant_rows(x.to(cuda), scale_dtype=torch.float32)
    qo, _, so = ops.quantize_rows(x.float().numpy(), "f32")
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


def test_quant_rows_near_ties_exact(cuda):
    """Values at and one ulp either side of half-integer multiples of the scale - where rounding x * (1/s) instead of
    the IEEE quotient x / s would pick the other integer - quantise exactly as clamp(rint(fp32(x / s)), -127, 127)
    (Int8Tensor.quantize, quant.py:37-41), over scales spanning 30 binades; fp32 rows, so any value is reachable."""
    rng = np.random.default_rng(5)
    M, K = 96, 4096
    x = np.empty((M, K), dtype=np.float32)
    for m in range(M):
        amax = np.float32(2.0 ** rng.integers(-20, 10)) * np.float32(rng.uniform(1, 2))
        s = np.float32(max(amax, np.float32(1e-8)) / np.float32(127))
        n = rng.integers(-127, 127, K).astype(np.float32) + np.float32(0.5)
        v = (n * s).astype(np.float32)
        k = rng.integers(-1, 2, K)
        v = np.where(k > 0, np.nextafter(v, np.float32(np.inf)), np.where(k < 0, np.nextafter(v, np.float32(-np.inf)), v))
        v[0] = amax
        x[m] = v
    xt = torch.from_numpy(x)
    q, sc = _lib.quant_rows(xt.to(cuda), scale_dtype=torch.float32)
    amax = np.abs(x).max(axis=1, keepdims=True)
    s_ref = (np.maximum(amax, np.float32(1e-8)) / np.float32(127)).astype(np.float32)
    q_ref = np.clip(np.rint((x / s_ref).astype(np.float32)), -127, 127).astype(np.int8)
    assert np.array_equal(sc.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


@pytest.mark.parametrize("M,K", [(5, 12288), (3, 9216), (7, 2048)])
def test_quant_rows_wide_rows(cuda, M, K):
    """Rows wider than one pass of the row's threads (several 8-value vectors per thread, ragged tails) against the
    fp32 formula."""
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(K)) * 3
    xb = x.to(torch.bfloat16)
    q, sc = _lib.quant_rows(xb.to(cuda), scale_dtype=torch.float32)
    xf = xb.float().numpy()
    s_ref = (np.maximum(np.abs(xf).max(axis=1, keepdims=True), np.float32(1e-8)) / np.float32(127)).astype(np.float32)
    q_ref = np.clip(np.rint((xf / s_ref).astype(np.float32)), -127, 127).astype(np.int8)
    assert np.array_equal(sc.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_quant_rows_smoothquant_and_stride(cuda):
    """SmoothedLinear's bf16(x * inv_s) before quantisation, on a row-strided view."""
    g = syn.gen(11)
    big = torch.randn(50, 1024, generator=g).to(torch.bfloat16)
    x = big[:, 256:768]
    inv_s = (torch.rand(512, generator=g) + 0.5).to(torch.bfloat16)
    q, s = _lib.quant_rows(big.to(cuda)[:, 256:768], scale_dtype=torch.float32, inv_s=inv_s.to(cuda))
    xs = ops.rbf(x.float().numpy() * inv_s.float().numpy())
    qo, _, so = ops.quantize_rows(xs, "f32")
    assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy(), so)


def test_dequant_rows(cuda, golden):
    q = torch.from_numpy(golden["kv.kq"]).reshape(-1, 128)
    s = from_bits(golden["kv.ks"], torch.float16).reshape(-1, 1)
    for dt, name in ((torch.bfloat16, "bf16"), (torch.float16, "f16"), (torch.float32, "f32")):
        y = _lib.dequant_rows(q.to(cuda), s.to(cuda), dt).cpu().float().numpy()
        ref = ops.dequantize_rows(q.numpy(), s.float().numpy(), name)
        assert np.array_equal(y, ref), name


def test_kv_append_golden(cuda, golden):
    """A6: the fp16 state's K/V appended in two slices at token offsets equal Int8Tensor.quantize byte for byte."""
    ac = syn.attn_case(S=2, T=160, rows=2, t=16, Hq=8, Hkv=2, D=128, seed=2)
    S, Hkv, T, D = ac.K16.shape
    kq = torch.zeros(S, Hkv, T, D, dtype=torch.int8, device=cuda)
    vq = torch.zeros_like(kq)
    ksc = torch.zeros(S, Hkv, T, dtype=torch.float16, device=cuda)
    vsc = torch.zeros_like(ksc)
    k = ac.K16.transpose(1, 2).to(cuda)                          # (S, T, Hkv, D) strided view of the cache layout
    v = ac.V16.transpose(1, 2).to(cuda)
    _lib.kv_append(k[:, :100], v[:, :100], kq, vq, ksc, vsc, t0=0)
    _lib.kv_append(k[:, 100:], v[:, 100:], kq, vq, ksc, vsc, t0=100)
    assert np.array_equal(kq.cpu().numpy(), golden["kv.kq"])
    assert np.array_equal(vq.cpu().numpy(), golden["kv.vq"])
    assert torch.equal(ksc.cpu().view(torch.int16).reshape(-1), torch.from_numpy(golden["kv.ks"]).reshape(-1))
    assert torch.equal(vsc.cpu().view(torch.int16).reshape(-1), torch.from_numpy(golden["kv.vs"]).reshape(-1))


@pytest.mark.parametrize("D", [64, 128, 256])
def test_kv_append_materialised_copy(cuda, D):
    """The kept bf16 copy written by the append equals materialize() of the int8 rows it wrote (oracle
    materialize_int8, bit for bit), at a token offset, leaving every other position of the copy untouched."""
    S, t, Hkv, T_cap, t0 = 3, 37, 2, 96, 50
    g = syn.gen(D)
    k = (torch.randn(S, t, Hkv, D, generator=g) * 2).to(torch.bfloat16).to(cuda)
    v = (torch.randn(S, t, Hkv, D, generator=g) * 0.3).to(torch.bfloat16).to(cuda)
    kq = torch.zeros(S, Hkv, T_cap, D, dtype=torch.int8, device=cuda)
    vq = torch.zeros_like(kq)
    ksc = torch.zeros(S, Hkv, T_cap, dtype=torch.bfloat16, device=cuda)
    vsc = torch.zeros_like(ksc)
    kb = torch.full((S, Hkv, T_cap, D), 7.0, dtype=torch.bfloat16, device=cuda)
    vb = torch.full_like(kb, 7.0)
    _lib.kv_append(k, v, kq, vq, ksc, vsc, t0=t0, kb=kb, vb=vb)
    for q8, sc, mat in ((kq, ksc, kb), (vq, vsc, vb)):
        want = ops.materialize_int8(q8[:, :, t0:t0 + t].cpu(), sc[:, :, t0:t0 + t, None].cpu())
        assert torch.equal(mat[:, :, t0:t0 + t].cpu().view(torch.int16), want.view(torch.int16))
        assert bool((mat[:, :, :t0] == 7.0).all()) and bool((mat[:, :, t0 + t:] == 7.0).all())
        # and the int8 rows are those of the append without the copy
    kq2, vq2, ksc2, vsc2 = (torch.zeros_like(x) for x in (kq, vq, ksc, vsc))
    _lib.kv_append(k, v, kq2, vq2, ksc2, vsc2, t0=t0)
    assert torch.equal(kq2, kq) and torch.equal(vq2, vq) and torch.equal(ksc2, ksc) and torch.equal(vsc2, vsc)


# ------------------------------------------------------------------------------------------------ norm + quant
@pytest.mark.parametrize("M,H", [(40, 256), (333, 4096)])
def test_rmsnorm_res_quant(cuda, M, H):
    g = syn.gen(M + H)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    res = (torch.randn(M, H, generator=g) * 3).to(torch.bfloat16)
    w = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    inv_s = (torch.rand(H, generator=g) + 0.5).to(torch.bfloat16)
    for use_s in (False, True):
        res_out = torch.empty(M, H, dtype=torch.bfloat16, device=cuda)
        y = torch.empty(M, H, dtype=torch.bfloat16, device=cuda)
        q, s = _lib.rmsnorm_res_quant(x.to(cuda), w.to(cuda), 1e-6, res_in=res.to(cuda), res_out=res_out,
                                      inv_s=inv_s.to(cuda) if use_s else None, y_out=y)
        h, yo, _, _ = ops.rmsnorm_res_quant(x.float().numpy(), w.float().numpy(), 1e-6, res=res.float().numpy(),
                                            inv_s=inv_s.float().numpy() if use_s else None)
        assert np.array_equal(res_out.cpu().float().numpy(), h)
        yk = y.cpu().float().numpy()
        # the sum of squares is reduced in a different order than torch's: y may differ by one bf16 ulp rarely
        assert np.mean(yk != yo) < 0.005 and np.all(np.abs(yk - yo) <= 2 ** -7 * np.abs(yo) + 1e-30)
        # the int8 bytes and scales are exactly the quantisation of the kernel's own normalised row
        qo, _, so = ops.quantize_rows(yk, "f32")
        assert np.array_equal(q.cpu().numpy(), qo) and np.array_equal(s.cpu().numpy(), so[:, 0])


def test_rmsnorm_golden(cuda, golden):
    g = syn.gen(3)
    x = torch.randn(40, 256, generator=g).to(torch.bfloat16)
    res_in = torch.randn(40, 256, generator=g).to(torch.bfloat16)
    nw = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    res_out = torch.empty(40, 256, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(40, 256, dtype=torch.bfloat16, device=cuda)
    _lib.rmsnorm_res_quant(x.to(cuda), nw.to(cuda), 1e-6, res_in=res_in.to(cuda), res_out=res_out, y_out=y,
                           want_q=False)
    assert torch.equal(res_out.cpu().view(torch.int16), from_bits(golden["norm.h"], torch.bfloat16).view(torch.int16))
    ref = from_bits(golden["norm.y"], torch.bfloat16).float()
    assert (y.cpu().float() != ref).float().mean() < 0.005


# ------------------------------------------------------------------------------------------------ W8A8 GEMM
def test_gemm_int32_golden(cuda, golden):
    a = torch.from_numpy(golden["quant.bf16.q"]).to(cuda)
    w = torch.from_numpy(golden["gemm.qweight"]).to(cuda)
    acc = _lib.gemm_w8a8(a, None, w, None, _lib.OD_EPI_INT32)
    assert np.array_equal(acc.cpu().numpy(), golden["gemm.acc"])


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (127, 512, 384), (300, 768, 1024), (1000, 1280, 2048),
                                   (1100, 512, 256), (2000, 256, 128), (1024, 1024, 640)])
def test_gemm_shapes_vs_oracle(cuda, M, N, K):
    """Single-CTA tiles (M < 1024) and CTA-pair tiles (M >= 1024, including row tails that leave the odd CTA's
    rows partly or wholly past M) against the int64 oracle: int32 accumulators and the bf16 epilogue bit for bit."""
    g = syn.gen(M + N + K)
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    sa = torch.rand(M, generator=g) * 0.01
    sw = (torch.rand(N, generator=g) * 0.01).to(torch.bfloat16)
    acc = _lib.gemm_w8a8(a.to(cuda), None, w.to(cuda), None, _lib.OD_EPI_INT32)
    ref = ops.gemm_i32(a.numpy(), w.numpy())
    assert np.array_equal(acc.cpu().numpy(), ref)
    y = _lib.gemm_w8a8(a.to(cuda), sa.to(cuda), w.to(cuda), sw.to(cuda), _lib.OD_EPI_BF16)
    yo = ops.gemm_w8a8_bf16(ref, sa.numpy(), sw.float().numpy())
    assert np.array_equal(y.cpu().float().numpy(), yo)


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (2048, 12288, 4096), (8192, 4096, 12288)])
def test_gemm_config2_int32_exact(cuda, M, N, K):
    """Config 2 shapes at full size: int32 accumulators equal cuBLASLt's exact int8 GEMM (torch._int_mm)."""
    gc = syn.gemm_case(M, N, K, seed=0)
    xq, sx = _lib.quant_rows(gc.x.to(cuda), scale_dtype=torch.float32)
    wq = gc.qweight.to(cuda)
    acc = _lib.gemm_w8a8(xq, None, wq, None, _lib.OD_EPI_INT32)
    ref = torch._int_mm(xq, wq.t())
    assert torch.equal(acc, ref)
    y = _lib.gemm_w8a8(xq, sx, wq, gc.wscale.to(cuda), _lib.OD_EPI_BF16)
    yo = ((ref.float() * sx.view(-1, 1)) * gc.wscale.to(cuda).float().view(1, -1)).to(torch.bfloat16)
    assert torch.equal(y, yo)


@pytest.mark.parametrize("M", [200, 1300])
def test_gemm_swiglu(cuda, M):
    g = syn.gen(5)
    F, K = 384, 512
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
    wg = torch.randint(-127, 128, (F, K), generator=g, dtype=torch.int8)
    wu = torch.randint(-127, 128, (F, K), generator=g, dtype=torch.int8)
    sa = torch.rand(M, generator=g) * 0.002
    sg = (torch.rand(F, generator=g) * 0.002).to(torch.bfloat16)
    su = (torch.rand(F, generator=g) * 0.002).to(torch.bfloat16)
    w = torch.from_numpy(ops.interleave_gate_up(wg.numpy(), wu.numpy()))
    s = torch.from_numpy(ops.interleave_gate_up(sg.float().numpy()[:, None], su.float().numpy()[:, None])[:, 0])
    y = _lib.gemm_w8a8(a.to(cuda), sa.to(cuda), w.to(cuda), s.to(torch.bfloat16).to(cuda), _lib.OD_EPI_SWIGLU)
    gq = ops.gemm_w8a8_bf16(ops.gemm_i32(a.numpy(), wg.numpy()), sa.numpy(), sg.float().numpy())
    uq = ops.gemm_w8a8_bf16(ops.gemm_i32(a.numpy(), wu.numpy()), sa.numpy(), su.float().numpy())
    ref = ops.silu_mul(gq, uq)
    yk = y.cpu().float().numpy()
    # exp() of two libraries may differ by an fp32 ulp: bf16 results equal except for rare one-ulp flips
    assert np.mean(yk != ref) < 0.01 and np.all(np.abs(yk - ref) <= 2 ** -7 * np.abs(ref) + 1e-6)


# ------------------------------------------------------------------------------------------------ small kernels
def test_embed(cuda, golden):
    qw = torch.from_numpy(golden["embed.qweight"]).to(cuda)
    sc = from_bits(golden["embed.scale"], torch.bfloat16).reshape(-1).to(cuda)
    g = syn.gen(3)
    for shape in [(40, 256), (40, 256), (256,)]:
        torch.randn(*shape, generator=g)
    torch.randn(24, 4 * 128 + 2 * 2 * 64, generator=g); torch.randn(64, generator=g); torch.randn(64, generator=g)
    torch.randint(0, 300, (24,), generator=g); torch.randn(24, 4 * 64, generator=g)
    torch.randn(100, 64, generator=g)
    ids = torch.randint(0, 100, (33,), generator=g)
    out = _lib.embed_i8(ids.to(cuda), qw, sc)
    assert torch.equal(out.cpu().view(torch.int16), from_bits(golden["embed.out"], torch.bfloat16).view(torch.int16))
    assert _lib.device_error() == 0


def test_qk_norm_rope_and_gate(cuda, golden):
    g = syn.gen(3)
    torch.randn(40, 256, generator=g); torch.randn(40, 256, generator=g); torch.randn(256, generator=g)
    Hq, Hkv, D, M = 4, 2, 64, 24
    qkv = torch.randn(M, Hq * 2 * D + 2 * Hkv * D, generator=g).to(torch.bfloat16)
    qw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16)
    kw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16)
    pos = torch.randint(0, 300, (M,), generator=g)
    cos, sin = ops.rope_tables(D, 1e6, 300)
    q, k, v = _lib.qk_norm_rope(qkv.to(cuda), pos.to(torch.int32).to(cuda), cos.to(cuda), sin.to(cuda), qw.to(cuda),
                                kw.to(cuda), 1e-6, Hq, Hkv, D)
    rq = from_bits(golden["rope.q"], torch.bfloat16).float()
    rk = from_bits(golden["rope.k"], torch.bfloat16).float()
    assert (q.cpu().float() != rq).float().mean() < 0.01
    assert (k.cpu().float() != rk).float().mean() < 0.01
    assert torch.allclose(q.cpu().float(), rq, atol=2e-2, rtol=0) and torch.allclose(k.cpu().float(), rk, atol=2e-2)
    assert torch.equal(v.cpu().float().reshape(M, -1), qkv[:, Hq * 2 * D + Hkv * D:].float())
    o = torch.randn(M, Hq * D, generator=g).to(torch.bfloat16)
    qo, so = _lib.gate_quant(o.to(cuda), qkv.to(cuda), Hq, D)
    gg, qr, sr = ops.gate_quant(o.float().numpy(), qkv.float().numpy(), Hq, D)
    ref = from_bits(golden["gate.g"], torch.bfloat16).float().numpy()
    assert np.mean(gg != ref) < 0.01
    # bytes equal the oracle's quantisation of the oracle's gated row wherever the gated row agrees
    assert np.mean(qo.cpu().numpy() != qr) < 0.01 and np.allclose(so.cpu().numpy(), sr, rtol=1e-2)


def test_readout(cuda, golden):
    logits = torch.from_numpy(golden["readout.logits"]).to(cuda)
    T = torch.from_numpy(golden["readout.T"]).to(cuda)
    mask = torch.from_numpy(golden["readout.mask"]).to(torch.uint8).to(cuda)
    nc = torch.from_numpy(golden["readout.none_col"]).to(cuda)
    p, ren, pn = _lib.readout(logits, T, mask, none_col=nc)
    assert np.allclose(p.cpu().numpy(), golden["readout.p"], atol=1e-6, rtol=0)
    assert np.allclose(ren.cpu().numpy(), golden["readout.renorm"], atol=1e-6, rtol=0)
    for i, c in enumerate(golden["readout.none_col"]):
        if c >= 0:
            assert abs(pn[i].item() - golden["readout.p"][i, c]) < 1e-6


# ------------------------------------------------------------------------------------------------ attention
def _attn_inputs(cuda, ac):
    Kq, Vq = ac.Kq.to(cuda), ac.Vq.to(cuda)
    ks, vs = ac.ks.reshape(ac.Kq.shape[:3]).to(cuda), ac.vs.reshape(ac.Kq.shape[:3]).to(cuda)
    return Kq, Vq, ks, vs


def test_prefix_attn_golden(cuda, golden):
    """A9: int8 prefix (with a left pad run and a hole on state 1) + causal own keys vs the reference's
    _split_attention. bf16 P.V rounding: the reference's own GPU test allows 2e-2 (tests/test_wide_attention.py)."""
    ac = syn.attn_case(S=2, T=160, rows=2, t=16, Hq=8, Hkv=2, D=128, seed=2)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    pm = torch.from_numpy(golden["attn.pm"])
    pmask = torch.stack([torch.ones_like(pm), pm]).to(torch.uint8).to(cuda)
    o, lse = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), 128 ** -0.5, Kp=Kq, Vp=Vq, ksc=ks,
                              vsc=vs, row_state=ac.row_state.to(cuda), pmask=pmask, want_lse=True)
    ref = from_bits(golden["attn.o"], torch.bfloat16).float()
    got = o.cpu().float()
    assert (got - ref).abs().max() < 2e-2
    assert (got - ref).norm() / ref.norm() < 5e-3
    # the same rows through p_lo (leading pads sliced, as the reference does) give the same result
    p_lo = torch.tensor([0, 7], dtype=torch.int32, device=cuda)
    o2 = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), 128 ** -0.5, Kp=Kq, Vp=Vq, ksc=ks, vsc=vs,
                          row_state=ac.row_state.to(cuda), pmask=pmask, p_lo=p_lo)
    assert (o2.cpu().float() - ref).abs().max() < 2e-2


def test_prefix_attn_row_order_invariant(cuda):
    """Every row sees the same key layout: permuting the rows permutes the outputs bit for bit."""
    ac = syn.attn_case(S=3, T=300, rows=5, t=12, Hq=32, Hkv=8, D=128, seed=7)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    perm = torch.randperm(ac.q.shape[0], generator=syn.gen(1))
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs)
    o = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), 128 ** -0.5, row_state=ac.row_state.to(cuda),
                         **args)
    op = _lib.prefix_attn(ac.q[perm].to(cuda), ac.k[perm].to(cuda), ac.v[perm].to(cuda), 128 ** -0.5,
                          row_state=ac.row_state[perm].to(cuda), **args)
    assert torch.equal(o[perm.to(cuda)], op)


def test_prefix_attn_question_level_and_causal(cuda):
    """Two-level prefix (state int8 + question bf16, right-padded questions) and a prefix-free causal pass, vs the
    oracle's split attention over the concatenated prefix (prefix_attn.py:94-99)."""
    g = syn.gen(9)
    S, T, Hq, Hkv, D, t = 2, 96, 4, 2, 64, 8
    ac = syn.attn_case(S=S, T=T, rows=3, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=9)
    NQ, Lq = 3, 20
    q_len = torch.tensor([20, 13, 5], dtype=torch.int32)
    q_state = torch.tensor([0, 1, 1])
    Kqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16)
    Vqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16)
    R = ac.q.shape[0]
    row_q = torch.tensor([0, 1, 2, 1, 0, 2][:R], dtype=torch.int32)
    row_state = q_state[row_q.long()].to(torch.int32)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    o = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), D ** -0.5, Kp=Kq, Vp=Vq, ksc=ks, vsc=vs,
                         row_state=row_state.to(cuda), Kq=Kqn.to(cuda), Vq=Vqn.to(cuda), row_q=row_q.to(cuda),
                         q_len=q_len.to(cuda)).cpu().float()
    Kp = ops.materialize_int8(ac.Kq, ac.ks)
    Vp = ops.materialize_int8(ac.Vq, ac.vs)
    for r in range(R):
        qr, s = int(row_q[r]), int(row_state[r])
        Kc = torch.cat([Kp[s], Kqn[qr].transpose(0, 1)], 1)
        Vc = torch.cat([Vp[s], Vqn[qr].transpose(0, 1)], 1)
        pm = torch.cat([torch.ones(T, dtype=torch.bool), torch.arange(Lq) < q_len[qr]])
        ref = ops.split_attention(ac.q[r:r + 1].transpose(1, 2), ac.k[r:r + 1].transpose(1, 2),
                                  ac.v[r:r + 1].transpose(1, 2), Kc, Vc, pm, D ** -0.5).transpose(1, 2)[0]
        assert (o[r] - ref).abs().max() < 2e-2, r
    # prefix-free causal attention (the state pass): rows of 200 tokens, no int8 prefix
    q = torch.randn(2, 200, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(2, 200, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(2, 200, Hkv, D, generator=g).to(torch.bfloat16)
    o = _lib.prefix_attn(q.to(cuda), k.to(cuda), v.to(cuda), D ** -0.5).cpu().float()
    rep = Hq // Hkv
    for r in range(2):
        qh, kh, vh = q[r].float().transpose(0, 1), k[r].float().transpose(0, 1), v[r].float().transpose(0, 1)
        sc = torch.einsum("htd,hsd->hts", qh, kh.repeat_interleave(rep, 0)) * D ** -0.5
        sc = sc.masked_fill(~torch.ones(200, 200, dtype=torch.bool).tril(), float("-inf"))
        ref = (torch.softmax(sc, -1) @ vh.repeat_interleave(rep, 0)).transpose(0, 1)
        assert (o[r] - ref).abs().max() < 2e-2


def test_prefix_attn_row_groups(cuda):
    """Rows of one question processed together in one tensor-core tile equal the rows processed alone (each row
    still attends only its own keys); groups of 1-3 rows, option rows of 5 tokens, 32 / 8 heads."""
    g = syn.gen(21)
    S, T, Hq, Hkv, D, t = 2, 200, 32, 8, 128, 5
    ac = syn.attn_case(S=S, T=T, rows=3, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=21)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    NQ, Lq = 2, 30
    Kqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    Vqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    row_q = torch.tensor([0, 0, 0, 1, 1, 1], dtype=torch.int32, device=cuda)
    q_len = torch.tensor([30, 17], dtype=torch.int32, device=cuda)
    own_hi = torch.tensor([5, 3, 4, 1, 5, 2], dtype=torch.int32, device=cuda)
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda), Kq=Kqn, Vq=Vqn, row_q=row_q,
                q_len=q_len, own_hi=own_hi)
    q, k, v = ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda)
    alone = _lib.prefix_attn(q, k, v, D ** -0.5, **args)
    groups = torch.tensor([[0, 3], [3, 2], [5, 1]], dtype=torch.int32, device=cuda)
    together = _lib.prefix_attn(q, k, v, D ** -0.5, row_groups=groups, max_group_rows=3, **args)
    for r in range(6):
        n = int(own_hi[r])
        assert (together[r, :n].float() - alone[r, :n].float()).abs().max() < 1e-2, r


def test_prefix_attn_group_spans_both_query_tiles(cuda):
    """A group of 4 option rows x 13 tokens x 4 heads (208 slots) fills both 128-slot query tiles of a CTA, one row
    straddling the tile boundary: every row equals the row processed alone, and the oracle."""
    g = syn.gen(23)
    S, T, Hq, Hkv, D, t = 2, 300, 32, 8, 128, 13
    ac = syn.attn_case(S=S, T=T, rows=4, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=23)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    R = ac.q.shape[0]
    own_hi = torch.tensor([13, 7, 12, 1, 13, 9, 4, 13][:R], dtype=torch.int32)
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda), own_hi=own_hi.to(cuda))
    q, k, v = ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda)
    alone = _lib.prefix_attn(q, k, v, D ** -0.5, **args)
    rs = ac.row_state.tolist()
    groups = [(i, 4) for i in range(0, R, 4)]
    assert all(len(set(rs[a:a + n])) == 1 for a, n in groups)
    together = _lib.prefix_attn(q, k, v, D ** -0.5, row_groups=torch.tensor(groups, dtype=torch.int32, device=cuda),
                                max_group_rows=4, **args)
    Kp = ops.materialize_int8(Kq.cpu(), ks.cpu()[..., None].to(torch.float16))
    Vp = ops.materialize_int8(Vq.cpu(), vs.cpu()[..., None].to(torch.float16))
    for r in range(R):
        n = int(own_hi[r])
        assert (together[r, :n].float() - alone[r, :n].float()).abs().max() < 1e-2, r
        s = rs[r]
        ref = ops.split_attention(ac.q[r:r + 1, :n].transpose(1, 2), ac.k[r:r + 1, :n].transpose(1, 2),
                                  ac.v[r:r + 1, :n].transpose(1, 2), Kp[s], Vp[s], None, D ** -0.5)
        assert (together[r:r + 1, :n].cpu().float() - ref.transpose(1, 2)).abs().max() < 2e-2, r


@pytest.mark.gpu
def test_prefix_attn_int8_dequant_exact(cuda):
    """One visible prefix key per state (p_hi = p_lo + 1, no own key visible): its softmax weight is exactly 1, so
    every output equals that key's dequantised V, bf16(vq * vs), bit for bit - the materialize() rounding of the
    reference (quant.py:43-45), over every int8 value and scales across many binades."""
    g = syn.gen(33)
    S, T, Hq, Hkv, D, t = 4, 256, 8, 2, 128, 3
    Vq = torch.randint(-128, 128, (S, Hkv, T, D), generator=g, dtype=torch.int8)
    Kq = torch.randint(-128, 128, (S, Hkv, T, D), generator=g, dtype=torch.int8)
    vs = (torch.rand(S, Hkv, T, generator=g) *
          torch.pow(2.0, torch.randint(-30, 10, (S, Hkv, T), generator=g).float())).to(torch.bfloat16)
    ks = torch.full((S, Hkv, T), 0.01).to(torch.bfloat16)
    row_state = torch.tensor([0, 1, 2, 3, 1], dtype=torch.int32)
    R = row_state.shape[0]
    p_lo = torch.tensor([0, 5, 100, 255], dtype=torch.int32)
    q = torch.randn(R, t, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(R, t, Hkv, D, generator=g).to(torch.bfloat16)
    zeros = torch.zeros(R, dtype=torch.int32, device=cuda)
    o = _lib.prefix_attn(q.to(cuda), k.to(cuda), k.to(cuda), D ** -0.5, Kp=Kq.to(cuda), Vp=Vq.to(cuda),
                         ksc=ks.to(cuda), vsc=vs.to(cuda), row_state=row_state.to(cuda), p_lo=p_lo.to(cuda),
                         p_hi=(p_lo + 1).to(cuda), own_lo=zeros, own_hi=zeros).cpu()
    deq = (Vq.float() * vs.float()[..., None]).to(torch.bfloat16)              # (S, Hkv, T, D)
    rep = Hq // Hkv
    for r in range(R):
        s = int(row_state[r])
        want = deq[s, :, int(p_lo[s]), :].repeat_interleave(rep, 0)           # (Hq, D)
        for i in range(t):
            assert torch.equal(o[r, i].view(torch.int16), want.view(torch.int16)), (r, i)


def test_dequant_rows_bf16_exact(cuda):
    """Int8Tensor.dequantize (quant.py:43-45) into bf16 with bf16 per-row scales (the KV-cache materialisation):
    every int8 value, scales over 40 binades, bit for bit against bf16(fp32(q) * fp32(s))."""
    g = torch.Generator().manual_seed(41)
    M, K = 1000, 128
    q = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    s = (torch.rand(M, 1, generator=g) * torch.pow(2.0, torch.randint(-30, 10, (M, 1), generator=g).float()))
    s = s.to(torch.bfloat16)
    y = _lib.dequant_rows(q.to(cuda), s.to(cuda), torch.bfloat16).cpu()
    ref = (q.float() * s.float()).to(torch.bfloat16)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


def test_prefix_attn_materialised_prefix_identical(cuda):
    """The state prefix given as the materialised bf16 cache (dequant_rows of the int8 cache, prefix_attn.py:146-149)
    produces bit-identical outputs and LSE to the int8 prefix dequantised inside the kernel: left pads, a hole,
    a question level and row groups."""
    g = syn.gen(57)
    S, T, Hq, Hkv, D, t = 2, 300, 32, 8, 128, 6
    ac = syn.attn_case(S=S, T=T, rows=4, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=57)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    ks, vs = ks.to(torch.bfloat16), vs.to(torch.bfloat16)           # the backbone's cache: bf16 scales
    Kb = _lib.dequant_rows(Kq.view(-1, D), ks.reshape(-1, 1), torch.bfloat16).view(Kq.shape)
    Vb = _lib.dequant_rows(Vq.view(-1, D), vs.reshape(-1, 1), torch.bfloat16).view(Vq.shape)
    pmask = torch.ones(S, T, dtype=torch.uint8)
    pmask[1, 40:77] = 0
    NQ, Lq = 2, 30
    Kqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    Vqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    R = ac.q.shape[0]
    row_q = torch.tensor([r % 2 for r in range(R)], dtype=torch.int32)
    order = torch.argsort(row_q * 16 + ac.row_state, stable=True)        # groups need shared state and question
    q, k, v = ac.q[order].to(cuda), ac.k[order].to(cuda), ac.v[order].to(cuda)
    rs, rq = ac.row_state[order].to(cuda), row_q[order].to(cuda)
    groups, i = [], 0
    while i < R:
        j = i
        while j < R and j - i < 2 and rs[j] == rs[i] and rq[j] == rq[i]:
            j += 1
        groups.append((i, j - i))
        i = j
    common = dict(row_state=rs, p_lo=torch.tensor([0, 9], dtype=torch.int32, device=cuda), pmask=pmask.to(cuda),
                  Kq=Kqn, Vq=Vqn, row_q=rq, q_len=torch.tensor([30, 11], dtype=torch.int32, device=cuda),
                  row_groups=torch.tensor(groups, dtype=torch.int32, device=cuda), max_group_rows=2, want_lse=True)
    o8, l8 = _lib.prefix_attn(q, k, v, D ** -0.5, Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, **common)
    ob, lb = _lib.prefix_attn(q, k, v, D ** -0.5, Kp=Kb, Vp=Vb, **common)
    assert torch.equal(o8, ob)
    assert torch.equal(l8, lb)


@pytest.mark.parametrize("nsplit", [2, 3, 5])
def test_prefix_attn_split_prefix_merges_exactly(cuda, nsplit):
    """The state prefix divided among several CTAs, partials merged by log-sum-exp: the same outputs and LSE as one
    CTA per tile (fp32 partials: within bf16 rounding), with a left-padded state, a question prefix and own keys."""
    g = syn.gen(31)
    S, T, Hq, Hkv, D, t = 2, 1000, 32, 8, 128, 3
    ac = syn.attn_case(S=S, T=T, rows=3, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=31)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    NQ, Lq = 2, 20
    Kqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    Vqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16).to(cuda)
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda),
                p_lo=torch.tensor([0, 77], dtype=torch.int32, device=cuda),
                p_hi=torch.tensor([1000, 905], dtype=torch.int32, device=cuda), Kq=Kqn, Vq=Vqn,
                row_q=torch.tensor([0, 1, 0, 1, 0, 1], dtype=torch.int32, device=cuda),
                q_len=torch.tensor([20, 9], dtype=torch.int32, device=cuda), want_lse=True)
    q, k, v = ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda)
    o1, l1 = _lib.prefix_attn(q, k, v, D ** -0.5, nsplit=1, **args)
    on, ln = _lib.prefix_attn(q, k, v, D ** -0.5, nsplit=nsplit, **args)
    assert _lib.device_error(cuda) == 0
    assert (o1.float() - on.float()).abs().max() < 1.6e-2
    assert (l1 - ln).abs().max() < 1e-4


def test_prefix_attn_plan_splits_small_launches(cuda):
    """A launch with fewer query tiles than SMs is split (one request, 8 KV heads, a 4096-token state); a full
    one is not."""
    ac = syn.attn_case(S=1, T=4096, rows=1, t=2, Hq=32, Hkv=8, D=128, seed=3)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    q, k, v = ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda)
    o = _lib.prefix_attn(q, k, v, 128 ** -0.5, Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda))
    o1 = _lib.prefix_attn(q, k, v, 128 ** -0.5, Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda),
                          nsplit=1)
    assert max(n for n, _ in _lib._PLANS.values()) > 1
    assert (o.float() - o1.float()).abs().max() < 1.6e-2


def _few_slot_case(scale_dtype, seed):
    """24 states x 2 groups (2 and 1 rows of 3 tokens, 32 / 8 heads: 24 and 12 query slots per group and KV head, the
    bandwidth-bound shape of a yes/no question), 300-token int8 states with left pads, an end (p_hi) and a hole, a
    right-padded question prefix and ragged own keys: 384 (group, KV head) tiles."""
    g = syn.gen(seed)
    S, T, Hq, Hkv, D, t = 24, 300, 32, 8, 128, 3
    ac = syn.attn_case(S=S, T=T, rows=3, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=seed)
    Kq, Vq, ks, vs = ac.Kq, ac.Vq, ac.ks.reshape(S, Hkv, T), ac.vs.reshape(S, Hkv, T)
    if scale_dtype == torch.bfloat16:                      # the backbone's cache: scales in the activation dtype
        ks, vs = ks.to(torch.bfloat16), vs.to(torch.bfloat16)
    R = S * 3
    p_lo = torch.randint(0, 40, (S,), generator=g, dtype=torch.int32)
    p_hi = T - torch.randint(0, 30, (S,), generator=g, dtype=torch.int32)
    pmask = torch.ones(S, T, dtype=torch.uint8)
    pmask[3, 100:180] = 0
    NQ, Lq = S, 20
    q_len = torch.randint(1, Lq + 1, (NQ,), generator=g, dtype=torch.int32)
    Kqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16)
    Vqn = torch.randn(NQ, Lq, Hkv, D, generator=g).to(torch.bfloat16)
    row_q = ac.row_state.clone()                           # one question per state
    own_hi = torch.randint(1, t + 1, (R,), generator=g, dtype=torch.int32)
    groups = [(3 * s + a, n) for s in range(S) for a, n in ((0, 2), (2, 1))]
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state, p_lo=p_lo, p_hi=p_hi, pmask=pmask, Kq=Kqn,
                Vq=Vqn, row_q=row_q, q_len=q_len, own_hi=own_hi)
    return ac, args, torch.tensor(groups, dtype=torch.int32), own_hi


def _few_slot_ref(ac, args, r):
    """Oracle for row r: the state prefix [p_lo, p_hi) with the hole, then the question's first q_len keys, then the
    row's own keys (causal, below own_hi)."""
    s, qr = int(args["row_state"][r]), int(args["row_q"][r])
    sd = args["ksc"].dtype
    Kp = ops.materialize_int8(args["Kp"][s], args["ksc"][s][..., None].to(sd))
    Vp = ops.materialize_int8(args["Vp"][s], args["vsc"][s][..., None].to(sd))
    T = Kp.shape[1]
    pm = (torch.arange(T) >= args["p_lo"][s]) & (torch.arange(T) < args["p_hi"][s]) & args["pmask"][s].bool()
    Lq = args["Kq"].shape[1]
    Kc = torch.cat([Kp, args["Kq"][qr].transpose(0, 1)], 1)
    Vc = torch.cat([Vp, args["Vq"][qr].transpose(0, 1)], 1)
    pm = torch.cat([pm, torch.arange(Lq) < args["q_len"][qr]])
    n = int(args["own_hi"][r])
    o = ops.split_attention(ac.q[r:r + 1, :n].transpose(1, 2), ac.k[r:r + 1, :n].transpose(1, 2),
                            ac.v[r:r + 1, :n].transpose(1, 2), Kc, Vc, pm, 128 ** -0.5)
    return o.transpose(1, 2)[0], n


@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.bfloat16])
def test_prefix_attn_few_slot_groups_vs_oracle(cuda, scale_dtype):
    """Groups of a few short rows (at most 24 query slots per KV head, one mostly empty query tile) against the
    oracle's split attention, with one CTA per state prefix and with the planned and an explicit split; the split
    results merge to the unsplit ones."""
    ac, args, groups, own_hi = _few_slot_case(scale_dtype, seed=61)
    dargs = {k: v.to(cuda) for k, v in args.items()}
    q, k, v = ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda)
    outs = {}
    for ns in (1, None, 3):
        o, lse = _lib.prefix_attn(q, k, v, 128 ** -0.5, row_groups=groups.to(cuda), max_group_rows=2, nsplit=ns,
                                  want_lse=True, **dargs)
        torch.cuda.synchronize()
        assert _lib.device_error(cuda) == 0
        outs[ns] = (o.cpu().float(), lse.cpu())
    o1, l1 = outs[1]
    for r in range(ac.q.shape[0]):
        ref, n = _few_slot_ref(ac, args, r)
        assert (o1[r, :n] - ref).abs().max() < 2e-2, r
    for ns in (None, 3):
        on, ln = outs[ns]
        for r in range(ac.q.shape[0]):
            n = int(own_hi[r])
            assert (on[r, :n] - o1[r, :n]).abs().max() < 1.6e-2, (ns, r)
            assert (ln[r, :, :n] - l1[r, :, :n]).abs().max() < 1e-4, (ns, r)


def test_prefix_attn_short_rows_row_order_invariant(cuda):
    """Rows of 3 tokens alone (12 query slots per KV head): permuting the rows permutes the outputs and LSE bit for
    bit."""
    ac = syn.attn_case(S=5, T=700, rows=7, t=3, Hq=32, Hkv=8, D=128, seed=67)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    perm = torch.randperm(ac.q.shape[0], generator=syn.gen(2))
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, want_lse=True)
    o, l = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), 128 ** -0.5,
                            row_state=ac.row_state.to(cuda), **args)
    op, lp = _lib.prefix_attn(ac.q[perm].to(cuda), ac.k[perm].to(cuda), ac.v[perm].to(cuda), 128 ** -0.5,
                              row_state=ac.row_state[perm].to(cuda), **args)
    assert torch.equal(o[perm.to(cuda)], op)
    assert torch.equal(l[perm.to(cuda)], lp)


def test_prefix_attn_fp16_dequant_exact(cuda):
    """As test_prefix_attn_int8_dequant_exact with fp16 scales (BASELINE config 3's cache): one visible prefix key
    per state, so each output is bf16(fp16(vq * vs)) bit for bit - over every int8 value and scales across the fp16
    range, subnormals included."""
    g = syn.gen(71)
    S, T, Hq, Hkv, D, t = 4, 256, 8, 2, 128, 3
    Vq = torch.randint(-128, 128, (S, Hkv, T, D), generator=g, dtype=torch.int8)
    Kq = torch.randint(-128, 128, (S, Hkv, T, D), generator=g, dtype=torch.int8)
    vs = (torch.rand(S, Hkv, T, generator=g) *
          torch.pow(2.0, torch.randint(-24, 8, (S, Hkv, T), generator=g).float())).to(torch.float16)
    ks = torch.full((S, Hkv, T), 0.01).to(torch.float16)
    row_state = torch.tensor([0, 1, 2, 3, 1], dtype=torch.int32)
    R = row_state.shape[0]
    p_lo = torch.tensor([0, 5, 100, 255], dtype=torch.int32)
    q = torch.randn(R, t, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(R, t, Hkv, D, generator=g).to(torch.bfloat16)
    zeros = torch.zeros(R, dtype=torch.int32, device=cuda)
    o = _lib.prefix_attn(q.to(cuda), k.to(cuda), k.to(cuda), D ** -0.5, Kp=Kq.to(cuda), Vp=Vq.to(cuda),
                         ksc=ks.to(cuda), vsc=vs.to(cuda), row_state=row_state.to(cuda), p_lo=p_lo.to(cuda),
                         p_hi=(p_lo + 1).to(cuda), own_lo=zeros, own_hi=zeros).cpu()
    deq = ops.materialize_int8(Vq, vs[..., None])                               # bf16(fp16(q * s))
    # an fp16 product that underflows is -0 for a negative q; a weighted sum started from +0 (here, as in the
    # reference's softmax(S) @ V) returns +0 there, so zeros compare without their sign
    deq = torch.where(deq == 0, torch.zeros_like(deq), deq)
    rep = Hq // Hkv
    for r in range(R):
        s = int(row_state[r])
        want = deq[s, :, int(p_lo[s]), :].repeat_interleave(rep, 0)
        for i in range(t):
            assert torch.equal(o[r, i].view(torch.int16), want.view(torch.int16)), (r, i)


@pytest.mark.parametrize("M,H,V", [(300, 256, 1000), (130, 4096, 4099), (7, 64, 256)])
def test_lm_logprob_matches_token_logprob(cuda, M, H, V):
    """Backbone.token_logprob on the tensor cores: bf16 logits, a vocabulary log-sum-exp (padded last tile left
    out), fp32 target logit. Within 5e-3 of the oracle (a bf16 logit may round the other way after a different
    summation order); splits of the vocabulary agree to fp32 rounding."""
    g = syn.gen(M + V)
    h = (torch.randn(M, H, generator=g) * 1.5).to(torch.bfloat16)
    w = torch.randn(V, H, generator=g) * 0.05
    qW, sW, _ = ops.quantize_rows(w.numpy(), "bf16")
    qW, sW = torch.from_numpy(qW), torch.from_numpy(sW[:, 0]).to(torch.bfloat16)
    Wb = (qW.to(torch.bfloat16) * sW[:, None])
    tok = torch.randint(0, V, (M,), generator=g)
    ref = ops.token_logprob(h, qW, sW, tok)
    args = [t.to(cuda) for t in (h, Wb, qW, sW, tok)]
    lp = _lib.lm_logprob(*args)
    assert (lp.cpu() - ref).abs().max() < 5e-3, (lp.cpu() - ref).abs().max()
    lp1 = _lib.lm_logprob(*args, vsplit=1)
    lp5 = _lib.lm_logprob(*args, vsplit=min(5, (V + 255) // 256))
    assert (lp1 - lp5).abs().max() < 1e-4
    assert _lib.device_error(cuda) == 0


@pytest.mark.parametrize("D,with_copy", [(128, True), (64, False)])
def test_qk_norm_rope_fused_kv_write_equals_kv_append(cuda, D, with_copy):
    """The fused cache write of od_qk_norm_rope_kv_i8 equals od_qk_norm_rope followed by od_kv_append_i8, byte for
    byte (int8 rows, bf16 scales, the materialised copy) at a token offset, with identical q / k / v outputs."""
    g = syn.gen(D + 7)
    S, t, Hq, Hkv, T_cap, t0 = 3, 21, 8, 2, 64, 30
    M = S * t
    qkv = (torch.randn(M, Hq * 2 * D + 2 * Hkv * D, generator=g) * 2).to(torch.bfloat16).to(cuda)
    pos = (t0 + torch.arange(t, dtype=torch.int32)).repeat(S).to(cuda)
    cos, sin = ops.rope_tables(D, 1e6, 256)
    qn = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    kn = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16).to(cuda)
    cos, sin = cos.to(cuda), sin.to(cuda)

    def cache():
        kq = torch.zeros(S, Hkv, T_cap, D, dtype=torch.int8, device=cuda)
        sc = torch.zeros(S, Hkv, T_cap, dtype=torch.bfloat16, device=cuda)
        mat = torch.zeros(S, Hkv, T_cap, D, dtype=torch.bfloat16, device=cuda) if with_copy else None
        return kq, kq.clone(), sc, sc.clone(), mat, (mat.clone() if with_copy else None)

    a = cache()
    q1, k1, v1 = _lib.qk_norm_rope(qkv, pos, cos, sin, qn, kn, 1e-6, Hq, Hkv, D)
    _lib.kv_append(k1.view(S, t, Hkv, D), v1.view(S, t, Hkv, D), a[0], a[1], a[2], a[3], t0=t0, kb=a[4], vb=a[5])
    b = cache()
    q2, k2, v2 = _lib.qk_norm_rope_kv(qkv, pos, cos, sin, qn, kn, 1e-6, Hq, Hkv, D, t, b[0], b[1], b[2], b[3], t0,
                                      kb=b[4], vb=b[5])
    assert torch.equal(q1, q2) and torch.equal(k1, k2) and torch.equal(v1, v2)
    for x, y in zip(a, b):
        if x is not None:
            assert torch.equal(x.view(torch.int8) if x.dtype == torch.int8 else x.view(torch.int16),
                               y.view(torch.int8) if y.dtype == torch.int8 else y.view(torch.int16))


def test_bounded_wait_reports_and_context_survives(cuda):
    """Failure detection on the GPU without a fault: a wait on a barrier nothing completes gives up after ~1 ms
    (2e6 cycles), the code lands in the device error word, od_device_error reads and clears it, and the next kernel
    runs normally."""
    assert _lib.device_error(cuda) == 0
    _lib.selftest_bounded_wait(2_000_000, cuda)
    assert _lib.device_error(cuda) == 0x7F0001
    assert _lib.device_error(cuda) == 0                       # read and cleared
    x = torch.randn(64, 256, generator=syn.gen(1)).to(torch.bfloat16).to(cuda)
    q, s = _lib.quant_rows(x, scale_dtype=torch.float32)
    qo, _, so = ops.quantize_rows(x.cpu().float().numpy(), "f32")
    assert np.array_equal(q.cpu().numpy(), qo)


@pytest.mark.parametrize("prefix", ["int8", "bf16"])
def test_prefix_attn_config3_full_shape(cuda, prefix):
    """BASELINE config 3 at its full per-request shape on 2 requests: a 4096-token int8 state (fp16 scales), 64
    option rows x 16 tokens, 32 / 8 heads, D 128, rows grouped 4 per CTA and the state prefix split as
    od_prefix_attn_plan chooses - against the oracle's _split_attention (prefix_attn.py:58-76, fp32). The prefix is
    read as int8 (dequantised in the kernel) or as the materialised bf16 cache. Tolerance: 2e-2 absolute, the
    reference's own GPU test bound for bf16 P.V; 5e-3 relative in norm."""
    S, T, rows, t, Hq, Hkv, D = 2, 4096, 64, 16, 32, 8, 128
    ac = syn.attn_case(S=S, T=T, rows=rows, t=t, Hq=Hq, Hkv=Hkv, D=D, seed=31)
    Kq, Vq, ks, vs = _attn_inputs(cuda, ac)
    Kp = ops.materialize_int8(ac.Kq, ac.ks)                       # (S, Hkv, T, D) bf16, as materialize() gives it
    Vp = ops.materialize_int8(ac.Vq, ac.vs)
    if prefix == "int8":
        kw = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs)
    else:
        kw = dict(Kp=Kp.to(cuda), Vp=Vp.to(cuda))
    per = 4                                                       # 4 rows x 16 tokens x 4 heads = 256 slots
    groups = torch.tensor([(a, per) for a in range(0, S * rows, per)], dtype=torch.int32, device=cuda)
    o = _lib.prefix_attn(ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), D ** -0.5, row_state=ac.row_state.to(cuda),
                         row_groups=groups, max_group_rows=per, **kw).cpu().float()
    torch.cuda.synchronize()
    assert _lib.device_error(cuda) == 0
    for s in range(S):
        for a in range(s * rows, (s + 1) * rows, 16):             # 16 rows at a time bound the CPU score tensor
            r = slice(a, a + 16)
            ref = ops.split_attention(ac.q[r].transpose(1, 2), ac.k[r].transpose(1, 2), ac.v[r].transpose(1, 2),
                                      Kp[s], Vp[s], None, D ** -0.5).transpose(1, 2)
            got = o[r]
            assert (got - ref).abs().max() < 2e-2, (s, a)
            assert (got - ref).norm() / ref.norm() < 5e-3, (s, a)


@pytest.mark.parametrize("M,N,K", [(512, 4096, 4096), (200, 768, 1024), (1000, 512, 1536), (1, 256, 512)])
def test_gemm_splitk_equals_unsplit(cuda, M, N, K):
    """Split-K (small M): the K range divided over 2..4 work items whose int32 partials a second kernel sums - bf16,
    SwiGLU and int32 epilogues identical to the unsplit GEMM, the int32 accumulators to the oracle's, twice in a
    row on the same workspace."""
    gc = syn.gemm_case(M=M, N=N, K=K, seed=6)
    xq, sx = _lib.quant_rows(gc.x.to(cuda), scale_dtype=torch.float32)
    W, sw = gc.qweight.to(cuda), gc.wscale.to(cuda).view(-1)
    ref32 = torch.from_numpy(ops.gemm_i32(xq.cpu().numpy(), gc.qweight.numpy()))
    for epi in (_lib.OD_EPI_BF16, _lib.OD_EPI_SWIGLU, _lib.OD_EPI_INT32):
        base = _lib.gemm_w8a8(xq, sx.view(-1), W, sw, epi, splits=1)
        for s in (2, 3, 4):
            if s > K // 128:
                continue
            for _ in range(2):
                got = _lib.gemm_w8a8(xq, sx.view(-1), W, sw, epi, splits=s)
                assert torch.equal(got, base), (epi, s)
        if epi == _lib.OD_EPI_INT32:
            assert torch.equal(base.cpu(), ref32)
    torch.cuda.synchronize()
    assert _lib.device_error(cuda) == 0
