"""CPU oracle of the V3 decision trunk - TEST INFRASTRUCTURE and part of the timed CPU baseline, never the product.

A PyTorch-CPU fp32 restatement of the reference's trunk (src/opendecider/v3.py): ScaleNorm (:43-50), the first-order
xATGLU (:53-67), interleaved-pair RoPE (:70-79), MHA through scaled_dot_product_attention with an additive float mask
(:82-100), V3Layer's self-attention / cross-attention / feed-forward (:116-130), and V3.forward's input projections,
CLS readout and score (:606-709) for the state-free branched-answer configuration, with the layer mix of
V3._mix_wide (:328-341). It reads the plan of opendecider_b200.v3.trunk_plan (the host-side layout of option and
question tokens, which the product uploads as it is).

Parity pin: tests/golden/e2e_config1.npz holds the reference's own decide_many logits on the seeded config-1
model; tests/test_oracle_e2e.py checks this trunk (inside oracle/model.py's OracleDecision) against them.
Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline, --impl reference) may import this module.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

NEG = -1e9   # masked logit (heads.py:13)


def _scalenorm(x, g, eps=1e-5):
    """ScaleNorm (v3.py:43-50): g * x / max(||x||, eps)."""
    return g * x / x.norm(dim=-1, keepdim=True).clamp_min(eps)


def _xatglu(p, prefix, x):
    """First-order xATGLU (v3.py:53-67): wo(g_a(wg x) * wv x), g_a(z) = ((atan z + pi/2) / pi)(1 + 2a) - a."""
    a = p[prefix + ".alpha"]
    z = F.linear(x, p[prefix + ".wg.weight"], p[prefix + ".wg.bias"])
    gate = (torch.atan(z) + math.pi / 2) / math.pi * (1 + 2 * a) - a
    return F.linear(gate * F.linear(x, p[prefix + ".wv.weight"], p[prefix + ".wv.bias"]), p[prefix + ".wo.weight"],
                    p[prefix + ".wo.bias"])


def _rope_pairs(x, pos):
    """Interleaved-pair RoPE of the trunk (v3.py:70-79), base 10000; pos (N, L) or None (= no rotation)."""
    if pos is None:
        return x
    dh = x.shape[-1]
    inv = 1.0 / (10000 ** (torch.arange(0, dh, 2, device=x.device, dtype=torch.float32) / dh))
    ang = pos.to(x.device).float()[:, None, :, None] * inv
    c, s = ang.cos().to(x.dtype), ang.sin().to(x.dtype)
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * c - x2 * s, x1 * s + x2 * c], -1).flatten(-2)


def _mha(p, prefix, h, x, ctx, bias, q_pos=None, k_pos=None):
    """MHA (v3.py:82-100): RoPE'd q/k, additive float mask, SDPA."""
    N, P, d = x.shape
    T = ctx.shape[1]
    dh = d // h
    q = _rope_pairs(F.linear(x, p[prefix + ".q.weight"]).view(N, P, h, dh).transpose(1, 2), q_pos)
    k = _rope_pairs(F.linear(ctx, p[prefix + ".k.weight"]).view(N, T, h, dh).transpose(1, 2), k_pos)
    v = F.linear(ctx, p[prefix + ".v.weight"]).view(N, T, h, dh).transpose(1, 2)
    o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    return F.linear(o.transpose(1, 2).reshape(N, P, d), p[prefix + ".o.weight"])


class OracleTrunk:
    """The decision trunk on the CPU in fp32. `params` under the reference V3 state-dict names; cfg a
    opendecider_b200.v3.TrunkConfig."""

    def __init__(self, cfg, params: dict):
        self.cfg = cfg
        self.p = {k: v.to(dtype=torch.float32) for k, v in params.items()}

    def prepare(self, q_lens, o_lens, n_opt, state_lens, up=None) -> dict:
        from opendecider_b200.v3 import trunk_plan
        return trunk_plan(q_lens, o_lens, n_opt, state_lens, up or (lambda x: x))

    def mix(self, f: torch.Tensor) -> torch.Tensor:
        """Softmax layer mix of multi-layer token features (V3._mix_wide, v3.py:328-341): (m, nL*d) -> (m, d)."""
        n, d = self.cfg.n_feat_layers, self.cfg.d_feat
        if n == 1:
            return f.float()
        w = torch.softmax(self.p["layer_mix"].float(), 0)
        return torch.einsum("l,mld->md", w, f.float().view(f.shape[0], n, d)).float()

    @torch.no_grad()
    def run(self, plan: dict, q_flat: torch.Tensor, o_flat: torch.Tensor, lp_flat: torch.Tensor | None = None):
        """V3.forward's trunk (v3.py:627-709): option/context stacks, decision layers, CLS readout, score.
        q_flat (sum lq, nL*d), o_flat (sum lo, nL*d) token features; lp_flat (sum lo,) the LM log-prob of each
        option token (lm_feature). Returns logits (N, K) fp32, NEG at pads."""
        p = self.p
        h, dm = self.cfg.n_heads, self.cfg.d_model
        N, K, P, Tc = plan["N"], plan["K"], plan["P"], plan["Tc"]
        opt_id, c_pad = plan["opt_id"], plan["c_pad"]
        x_pad = opt_id < 0
        same = ((opt_id[:, :, None] == opt_id[:, None, :]) & ~x_pad[:, :, None]).float()
        b_cross = torch.zeros(c_pad.shape).masked_fill(c_pad, NEG)[:, None, None, :]
        own = opt_id[:, None, :] == torch.arange(K)[None, :, None]
        b_cls = torch.zeros(own.shape).masked_fill(~own, NEG)[:, None]
        # the input projections on the real tokens, scattered into the padded layouts; a padding row (zeros in the
        # reference) projects to the bias alone: proj_option's for option pads, proj_state's for context pads
        x = p["proj_option.bias"].expand(N, P, dm).clone()
        x[plan["rc"]] = F.linear(_scalenorm(self.mix(o_flat), p["in_norm.g"]), p["proj_option.weight"],
                                 p["proj_option.bias"])
        lpX = None
        if self.cfg.lm_feature:             # token-level log-prob feature (v3.py:666-672)
            lpX = torch.zeros(N, P)
            lpX[plan["rc"]] = lp_flat.float()
            x = x + F.linear(lpX[..., None], p["lp_proj.weight"], p["lp_proj.bias"])
        c = p["proj_state.bias"].expand(N, Tc, dm).clone()
        c[plan["qrc"]] = F.linear(_scalenorm(self.mix(q_flat), p["in_norm.g"]), p["proj_question.weight"],
                                  p["proj_question.bias"])
        opos, cpos = plan["opos"], plan["cpos"]
        for i in range(self.cfg.decision_layers):
            L = f"layers.{i}."
            b_self = p[L + "same_bias"].view(1, h, 1, 1) * same[:, None]
            b_self = b_self.masked_fill(x_pad[:, None, None, :], NEG)
            hx = _scalenorm(x, p[L + "n1.g"])
            x = x + _mha(p, L + "self_attn", h, hx, hx, b_self, opos, opos)
            x = x + _mha(p, L + "cross", h, _scalenorm(x, p[L + "n2.g"]), _scalenorm(c, p[L + "n2c.g"]),
                         b_cross, None, cpos)
            x = x + _xatglu(p, L + "ff", _scalenorm(x, p[L + "n3.g"]))
        hc = p["cls.weight"].expand(N, K, dm)
        hc = hc + _mha(p, "cls_attn", h, _scalenorm(hc, p["cls_nq.g"]), _scalenorm(x, p["cls_nkv.g"]),
                       b_cls, None, opos)
        hc = hc + _xatglu(p, "cls_ff", _scalenorm(hc, p["cls_nf.g"]))
        hc = _scalenorm(hc, p["final_norm.g"])
        logits = F.linear(hc, p["score.weight"], p["score.bias"]).squeeze(-1).float()
        if lpX is not None:                 # gated skip of the length-normalised log-likelihood (v3.py:702-706)
            own_f = own.float()
            ll = (own_f * lpX[:, None, :]).sum(-1) / own_f.sum(-1).clamp_min(1)
            logits = logits + p["lm_skip"] * ll
        return logits.masked_fill(~plan["opt_mask"], NEG)
