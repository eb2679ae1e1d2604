"""CPU oracle of the decision forward pass's operators - TEST INFRASTRUCTURE, never the product path.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may import this module,
and only as the checker or the timed CPU baseline. Each function restates the reference algorithm in numpy (integer
and byte work, bit-exact) or PyTorch CPU float32 (floating-point work), citing the reference file:line it follows.
The rounding points of bf16 tensors are emulated with `rbf` (round to nearest even through bfloat16), matching how
PyTorch computes a bf16 elementwise op (in fp32, one rounding of the result).

Parity pins: tests/test_oracle_golden.py checks these functions against tests/golden/*.npz, which
tests/golden/make_golden.py produced by running the reference implementation itself (src/opendecider) on the same
seeded inputs.
"""
from __future__ import annotations

import numpy as np
import torch

F32 = np.float32


# ------------------------------------------------------------------------------------------------ rounding helpers
def rbf(x) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest even) and back to float32."""
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=F32))
    return t.to(torch.bfloat16).float().numpy()


def rhf(x) -> np.ndarray:
    """Round float32 values to float16 (nearest even) and back to float32."""
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def round_to(x, dtype: str) -> np.ndarray:
    return {"bf16": rbf, "f16": rhf, "f32": lambda v: np.asarray(v, dtype=F32)}[dtype](x)


# ------------------------------------------------------------------------------------------------ A1 / A5 / A6
def quantize_rows(x, scale_dtype: str = "f32"):
    """Int8Tensor.quantize (src/opendecider/quant.py:37-41) over the last dim; Int8Linear's weight quantiser is the
    same formula (quant.py:124-127). x holds float32 values (the `.float()` of the input). Returns
    (q int8, stored scale as float32 values after rounding to scale_dtype, fp32 scale used for q)."""
    xf = np.asarray(x, dtype=F32)
    amax = np.abs(xf).max(-1, keepdims=True)
    s = np.maximum(amax, F32(1e-8)) / F32(127.0)
    q = np.clip(np.rint(xf / s), -127, 127).astype(np.int8)
    return q, round_to(s, scale_dtype), s


def dequantize_rows(q, scale, dtype: str = "bf16"):
    """Int8Tensor.dequantize (quant.py:43-45): q.to(dt) * scale.to(dt), rounded to dt."""
    s = round_to(scale, dtype)
    return round_to(q.astype(F32) * s, dtype)


# ------------------------------------------------------------------------------------------------ A2
def gemm_i32(a_q, w_q) -> np.ndarray:
    """int32 accumulators of the W8A8 GEMM: sum_k A[m,k] W[n,k] (exact; the int64 product never overflows)."""
    return (a_q.astype(np.int64) @ w_q.astype(np.int64).T).astype(np.int32)


def gemm_w8a8_bf16(acc, sa, sw):
    """Dequant epilogue: bf16((float(acc) * s_x[m]) * s_w[n]); s_x fp32 per token, s_w the bf16 weight scale."""
    return rbf((acc.astype(F32) * np.asarray(sa, F32).reshape(-1, 1)) * np.asarray(sw, F32).reshape(1, -1))


def silu_mul(g, u):
    """Qwen3_5MLP.forward's act_fn(gate) * up on bf16 tensors (site-packages transformers
    models/qwen3_5/modeling_qwen3_5.py:706-708): SiLU in fp32 rounded to bf16, product rounded to bf16."""
    g = np.asarray(g, F32)
    a = rbf(g / (F32(1.0) + np.exp(-g)))
    return rbf(a * np.asarray(u, F32))


def interleave_gate_up(w_gate, w_up, block: int = 128):
    """Row order of the fused gate/up weight the SwiGLU epilogue reads: blocks of `block` gate rows then the same
    `block` up rows (an internal layout of this implementation, built from the reference's two Int8Linear weights)."""
    F = w_gate.shape[0]
    assert F % block == 0
    parts = []
    for b in range(0, F, block):
        parts += [w_gate[b:b + block], w_up[b:b + block]]
    return np.concatenate(parts, 0)


# ------------------------------------------------------------------------------------------------ A3 + A4 + A5
def rmsnorm(h, w, eps):
    """Qwen3_5RMSNorm.forward (modeling_qwen3_5.py:720-725) on bf16 values: float32 math, (1 + w), one rounding."""
    hf = torch.from_numpy(np.asarray(h, F32))
    var = hf.pow(2).mean(-1, keepdim=True)
    out = hf * torch.rsqrt(var + eps)
    out = out * (1.0 + torch.from_numpy(np.asarray(w, F32)))
    return rbf(out.numpy())


def rmsnorm_res_quant(x, w, eps, res=None, inv_s=None):
    """Decoder pre-norm block: h = bf16(res + x) (modeling_qwen3_5.py:768/781), y = RMSNorm(h), optional
    SmoothedLinear multiply bf16(y * inv_s) (quant.py:328-329), then per-token int8 with fp32 scales.
    Returns (h, y, q, s)."""
    h = np.asarray(x, F32) if res is None else rbf(np.asarray(res, F32) + np.asarray(x, F32))
    y = rmsnorm(h, w, eps)
    if inv_s is not None:
        y = rbf(y * np.asarray(inv_s, F32))
    q, _, s = quantize_rows(y, "f32")
    return h, y, q, s[..., 0]


# ------------------------------------------------------------------------------------------------ attention pieces
def rope_tables(D: int, theta: float, n_pos: int, dtype=torch.bfloat16):
    """cos/sin tables of Qwen3_5TextRotaryEmbedding (modeling_qwen3_5.py:85-155) for text positions 0..n_pos-1 with
    partial_rotary_factor 1.0: inv_freq = 1 / theta^(arange(0, D, 2) / D), emb = cat(freqs, freqs), cast to dtype."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(dtype=torch.float) / D))
    pos = torch.arange(n_pos, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def qk_norm_rope(qkv, pos, cos, sin, qw, kw, eps, Hq, Hkv, D):
    """Qwen3_5Attention.forward (modeling_qwen3_5.py:647-662) on bf16 values for a flat token batch: gated q split,
    per-head RMSNorm, apply_rotary_pos_emb (:544-573) with bf16 products and sum. Returns q, k, v (M, H, D)."""
    qkv = np.asarray(qkv, F32)
    M = qkv.shape[0]
    qg = qkv[:, : Hq * 2 * D].reshape(M, Hq, 2 * D)
    q = qg[..., :D]
    k = qkv[:, Hq * 2 * D: Hq * 2 * D + Hkv * D].reshape(M, Hkv, D)
    v = qkv[:, Hq * 2 * D + Hkv * D:].reshape(M, Hkv, D)
    q = rmsnorm(q, qw, eps)
    k = rmsnorm(k, kw, eps)
    c = cos.float().numpy()[pos][:, None, :]
    s = sin.float().numpy()[pos][:, None, :]

    def rot(x):
        rh = np.concatenate([-x[..., D // 2:], x[..., : D // 2]], -1)
        return rbf(rbf(x * c) + rbf(rh * s))

    return rot(q), rot(k), v.copy()


def gate_quant(o, qkv, Hq, D):
    """o * sigmoid(gate) on bf16 values (modeling_qwen3_5.py:666-667), then per-token int8 (fp32 scales)."""
    M = o.shape[0]
    gate = np.asarray(qkv, F32)[:, : Hq * 2 * D].reshape(M, Hq, 2 * D)[..., D:].reshape(M, Hq * D)
    sg = rbf(F32(1.0) / (F32(1.0) + np.exp(-gate)))
    g = rbf(np.asarray(o, F32).reshape(M, -1) * sg)
    q, _, s = quantize_rows(g, "f32")
    return g, q, s[..., 0]


def split_attention(q, k, v, Kp, Vp, pm, scale):
    """prefix_attn._split_attention's CPU branch (src/opendecider/prefix_attn.py:58-76): rows' queries q (n, Hq, t, D)
    attend the shared prefix Kp/Vp (Hkv, T, D) (pm (T,) bool real keys or None) and their own k/v (n, Hkv, t, D)
    causally, merged exactly by log-sum-exp. float32 torch tensors in, (n, Hq, t, D) float32 out."""
    n, Hq, t, D = q.shape
    Hkv, T = Kp.shape[0], Kp.shape[1]
    g = Hq // Hkv
    Ke, Ve = Kp.repeat_interleave(g, 0).float(), Vp.repeat_interleave(g, 0).float()
    sp = torch.einsum("nhtd,hsd->nhts", q.float(), Ke) * scale
    if pm is not None:
        sp = sp.masked_fill(~pm.view(1, 1, 1, T), float("-inf"))
    l_p = torch.logsumexp(sp, -1)
    o_p = torch.softmax(sp, -1) @ Ve
    so = torch.einsum("nhtd,nhud->nhtu", q.float(), k.repeat_interleave(g, 1).float()) * scale
    so = so.masked_fill(~torch.ones(t, t, dtype=torch.bool).tril(), float("-inf"))
    l_o = torch.logsumexp(so, -1)
    o_o = torch.softmax(so, -1) @ v.repeat_interleave(g, 1).float()
    m = torch.maximum(l_p, l_o)
    wp, wo = torch.exp(l_p - m), torch.exp(l_o - m)
    return (o_p * wp[..., None] + o_o * wo[..., None]) / (wp + wo)[..., None]


def materialize_int8(q, scale, dtype=torch.bfloat16):
    """materialize(Int8Tensor) (quant.py:112-115 -> :43-45) then .to(dtype) as shared_prefix_attention does
    (prefix_attn.py:147-148): q.to(s.dtype) * s in the scale's dtype, then cast."""
    sd = scale.dtype
    return (q.to(sd) * scale.to(sd)).to(dtype)


# ------------------------------------------------------------------------------------------------ A13
def readout(logits, T, mask, bias=None, none_col=None):
    """Decider._probs' readout (src/opendecider/decider.py:255-257) and _normalize (:26-29):
    p = softmax(logits / T + bias) * mask; renorm = clamp(p, 0) / sum over the caller's options, in float64."""
    lg = torch.as_tensor(logits, dtype=torch.float32)
    Tt = torch.as_tensor(T, dtype=torch.float32).reshape(-1, 1)
    z = lg / Tt + (torch.zeros_like(lg) if bias is None else torch.as_tensor(bias, dtype=torch.float32))
    p = torch.softmax(z, -1) * torch.as_tensor(mask).to(torch.float32)
    N, K = p.shape
    renorm = torch.zeros(N, K, dtype=torch.float64)
    p_none = torch.zeros(N, dtype=torch.float32)
    for i in range(N):
        kc = K if none_col is None or int(none_col[i]) < 0 else int(none_col[i])
        pd = p[i, :kc].double().clamp_min(0)
        renorm[i, :kc] = pd / pd.sum()
        if none_col is not None and int(none_col[i]) >= 0:
            p_none[i] = p[i, int(none_col[i])]
    return p.numpy(), renorm.numpy(), p_none.numpy()


# ------------------------------------------------------------------------------------------------ (f.2) LM head
def token_logprob(h, qW, sW, tok):
    """Backbone.token_logprob (src/opendecider/backbone.py:165-178) with the tied int8 head (Int8Embedding.dequant_
    rows, quant.py:202-203): logits = bf16(bf16(h) @ bf16(q * s)^T) as the reference's bf16 matmul returns them,
    log-sum-exp over the vocabulary in fp32 (its chunked logaddexp is the same sum), the target logit in fp32 from
    q.float() * s.float(). h (M, H) bf16, qW (V, H) int8, sW (V,) or (V, 1) bf16, tok (M,) long -> (M,) fp32."""
    s = sW.reshape(-1, 1)
    Wb = qW.to(torch.bfloat16) * s.to(torch.bfloat16)
    hb = h.to(torch.bfloat16)
    lse = torch.logsumexp((hb @ Wb.t()).float(), dim=-1)
    target = (h.float() * (qW[tok].float() * s[tok].float())).sum(-1)
    return target - lse
