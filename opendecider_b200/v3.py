"""Branched option rows and the V3 decision trunk: backbone features -> one logit per option.

Row passes (the hot part, all in libod_b200 through Backbone.run):
  branched_feats_qcache   V3._branched_feats_qcache (src/opendecider/v3.py:446-534): ONE right-padded question pass
                          over [question + canonical listing + "Answer:"] continuing each question's state (int8
                          prefix, captured bf16 question K/V), then option rows carrying only their own answer tokens,
                          attending [state int8 ; question bf16 ; own causal] in one kernel call per layer. Rows are
                          sorted by option length and run in chunks as wide as their longest option.
  branched_feats          V3._branched_feats (v3.py:393-444): one row [question ; option] per option continuing the
                          state, used below the question-cache threshold (decider.QCACHE_MIN_ROWS).
Trunk (small, d_model 512): V3.forward (v3.py:606-709) with the serving configuration of the shipped 9B checkpoint
(v3_cross="question" so the trunk never reads state tokens, slot_emb="none", readout "last", no context layers) and
a softmax layer mix of the multi-layer features. It runs as PyTorch fp32 ops on the GPU (cuBLAS for its small
GEMMs); its parameter names are the reference V3's, so a reference checkpoint's trunk loads unchanged.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .backbone import Backbone, KVCache, PassSpec
from .batching import answer_option_text, answer_row_prefix, segment_layout

NEG = -1e9   # masked logit (heads.py:13)


# ------------------------------------------------------------------------------------------------ trunk
@dataclass
class TrunkConfig:
    d_feat: int                 # backbone hidden size
    n_feat_layers: int          # feature layers mixed per token
    d_model: int = 512
    n_heads: int = 8
    decision_layers: int = 4


def _lin(g, out_f, in_f, bias=True):
    b = 1.0 / math.sqrt(in_f)       # torch.nn.Linear's default init bounds
    w = (torch.rand(out_f, in_f, generator=g) * 2 - 1) * b
    return (w, (torch.rand(out_f, generator=g) * 2 - 1) * b) if bias else (w, None)


def trunk_state_dict(cfg: TrunkConfig, seed: int = 0) -> dict:
    """Seeded random trunk parameters under the reference V3's state-dict names. Linears use PyTorch's default init
    bounds; the ScaleNorm gains start at sqrt(d) and the xATGLU alphas, same-option biases and the layer mix get
    small random values so every term of the forward is exercised."""
    g = torch.Generator().manual_seed(seed)
    d, dm, h = cfg.d_feat, cfg.d_model, cfg.n_heads
    ff = int(round(dm * (8 / 3) / 8)) * 8
    sd = {}

    def put(name, w, b=None):
        sd[name + ".weight"] = w
        if b is not None:
            sd[name + ".bias"] = b

    sd["layer_mix"] = torch.randn(cfg.n_feat_layers, generator=g) * 0.5
    sd["in_norm.g"] = torch.tensor(math.sqrt(d))
    for n in ("proj_state", "proj_question", "proj_option"):
        put(n, *_lin(g, dm, d))

    def mha(prefix):
        for n in ("q", "k", "v", "o"):
            put(f"{prefix}.{n}", *_lin(g, dm, dm, bias=False))

    def xatglu(prefix):
        put(prefix + ".wg", *_lin(g, ff, dm))
        put(prefix + ".wv", *_lin(g, ff, dm))
        put(prefix + ".wo", *_lin(g, dm, ff))
        sd[prefix + ".alpha"] = torch.randn((), generator=g) * 0.1

    for i in range(cfg.decision_layers):
        p = f"layers.{i}."
        for n in ("n1", "n2", "n2c", "n3"):
            sd[p + n + ".g"] = torch.tensor(math.sqrt(dm))
        mha(p + "self_attn")
        mha(p + "cross")
        xatglu(p + "ff")
        sd[p + "same_bias"] = torch.randn(h, generator=g) * 0.5
    sd["cls.weight"] = torch.randn(1, dm, generator=g)
    for n in ("cls_nq", "cls_nkv", "cls_nf", "final_norm"):
        sd[n + ".g"] = torch.tensor(math.sqrt(dm))
    mha("cls_attn")
    xatglu("cls_ff")
    put("score", *_lin(g, 1, dm))
    put("rel", *_lin(g, 1, dm))
    return sd


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


class V3Trunk:
    """The decision trunk on the GPU (fp32). `params` under the reference V3 state-dict names."""

    def __init__(self, cfg: TrunkConfig, params: dict, device):
        self.cfg = cfg
        self.p = {k: v.to(device=device, dtype=torch.float32) for k, v in params.items()}
        self.device = torch.device(device)

    def mix(self, f: torch.Tensor) -> torch.Tensor:
        """Softmax layer mix of multi-layer token features (V3._mix_wide, v3.py:328-341): (m, nL*d) -> (m, d)."""
        n, d = self.cfg.n_feat_layers, self.cfg.d_feat
        if n == 1:
            return f.float()
        w = torch.softmax(self.p["layer_mix"].float(), 0)
        return torch.einsum("l,mld->md", w, f.float().view(f.shape[0], n, d)).float()

    @torch.no_grad()
    def forward(self, q_flat, q_lens, o_flat, o_lens, n_opt, opt_mask, state_lens):
        """V3.forward (v3.py:606-709) for the state-free trunk. q_flat (sum lq, nL*d) question-token features,
        o_flat (sum lo, nL*d) option-token features; q_lens/o_lens/n_opt/state_lens CPU longs (state_lens = the
        state length of each question's state); opt_mask (N, K) bool on the device. Returns logits (N, K) fp32."""
        p, dev = self.p, self.device
        h, dm, df = self.cfg.n_heads, self.cfg.d_model, self.cfg.d_feat
        N, K = opt_mask.shape
        opt_q = torch.repeat_interleave(torch.arange(N), n_opt)
        opt_k = torch.arange(int(n_opt.sum())) - torch.repeat_interleave(torch.cumsum(n_opt, 0) - n_opt, n_opt)
        # ---- options -> (N, P, d)
        row, col, seg, pos, row_len = segment_layout(o_lens, opt_q, N)
        P = int(row_len.max())
        rc = (row.to(dev), col.to(dev))
        X = torch.zeros(N, P, df, device=dev)
        X[rc] = self.mix(o_flat)
        opt_id = torch.full((N, P), -1, dtype=torch.long, device=dev)
        opt_id[rc] = opt_k[seg].to(dev)
        opos = torch.zeros(N, P, dtype=torch.long, device=dev)
        opos[rc] = pos.to(dev)
        x_pad = opt_id < 0
        # ---- context = question tokens only, positioned after the state (state-free trunk)
        Tc = int(q_lens.max())
        C = torch.zeros(N, Tc, df, device=dev)
        qrow, qcol, _, _, _ = segment_layout(q_lens, torch.arange(N), N)
        C[(qrow.to(dev), qcol.to(dev))] = self.mix(q_flat)
        t = torch.arange(Tc)[None, :]
        in_q = t < q_lens[:, None]
        cpos = (t + state_lens[:, None]).to(dev)
        c_pad = (~in_q).to(dev)
        C = C * (~c_pad)[..., None]
        # ---- stack inputs
        x = F.linear(_scalenorm(X, p["in_norm.g"]), p["proj_option.weight"], p["proj_option.bias"])
        cin = _scalenorm(C, p["in_norm.g"])
        c = torch.where(in_q.to(dev)[..., None], F.linear(cin, p["proj_question.weight"], p["proj_question.bias"]),
                        F.linear(cin, p["proj_state.weight"], p["proj_state.bias"]))
        same = (opt_id[:, :, None] == opt_id[:, None, :]) & ~x_pad[:, :, None]
        b_cross = torch.zeros(c_pad.shape, device=dev).masked_fill(c_pad, NEG)[:, None, None, :]
        for i in range(self.cfg.decision_layers):
            L = f"layers.{i}."
            b_self = p[L + "same_bias"].view(1, h, 1, 1) * same[:, None].float()
            b_self = b_self.masked_fill(x_pad[:, None, None, :], NEG)
            hx = _scalenorm(x, p[L + "n1.g"])
            x = x + _mha(p, L + "self_attn", h, hx, hx, b_self, opos, opos)
            x = x + _mha(p, L + "cross", h, _scalenorm(x, p[L + "n2.g"]), _scalenorm(c, p[L + "n2c.g"]), b_cross,
                         None, cpos)
            x = x + _xatglu(p, L + "ff", _scalenorm(x, p[L + "n3.g"]))
        # ---- CLS readout: one query per option attends only to that option's tokens
        own = opt_id[:, None, :] == torch.arange(K, device=dev)[None, :, None]
        b = torch.zeros(own.shape, device=dev).masked_fill(~own, NEG)[:, None]
        hc = p["cls.weight"].expand(N, K, dm)
        hc = hc + _mha(p, "cls_attn", h, _scalenorm(hc, p["cls_nq.g"]), _scalenorm(x, p["cls_nkv.g"]), b, None, opos)
        hc = hc + _xatglu(p, "cls_ff", _scalenorm(hc, p["cls_nf.g"]))
        hc = _scalenorm(hc, p["final_norm.g"])
        logits = F.linear(hc, p["score.weight"], p["score.bias"]).squeeze(-1).float()
        return logits.masked_fill(~opt_mask, NEG)


# ------------------------------------------------------------------------------------------------ row passes
def _rect(tok_lists, pad_id, width=None):
    lens = torch.tensor([len(t) for t in tok_lists], dtype=torch.long)
    L = width or max(1, int(lens.max()))
    ids = torch.full((len(tok_lists), L), pad_id, dtype=torch.long)
    for i, t in enumerate(tok_lists):
        ids[i, : len(t)] = torch.tensor(t, dtype=torch.long)
    return ids, lens


def branched_feats_qcache(bb: Backbone, tok, questions, cache: KVCache, list_cap: int = 16, chunk: int = 4096):
    """Question cache path (v3.py:446-534). Returns (q_flat, lq, o_flat, lo): features of every question token and
    every option token in question / option order, (tokens, nL*H) bf16 on the device; lengths on the CPU."""
    dev, feats = bb.device, bb.cfg.feature_layers
    N = len(questions)
    q_tok = tok([answer_row_prefix(q.prompt, q.options, list_cap) for q in questions],
                add_special_tokens=False)["input_ids"]
    o_tok = tok([answer_option_text(o) for q in questions for o in q.options], add_special_tokens=False)["input_ids"]
    n_opt = torch.tensor([len(q.options) for q in questions])
    row_q = torch.repeat_interleave(torch.arange(N), n_opt)
    Qids, lq = _rect(q_tok, bb.pad_id)
    Lq = Qids.shape[1]
    sidx = torch.tensor([q.state_idx for q in questions], dtype=torch.int32)
    T = cache.T
    # ---- question pass: right-padded, continuing each question's state (positions T + j)
    qpos = (T + torch.arange(Lq, dtype=torch.int32)).expand(N, Lq)
    spec = PassSpec(ids=Qids.to(dev), pos=qpos.to(dev), own_hi=lq.to(torch.int32).to(dev), cache=cache,
                    row_state=sidx.to(dev), capture=True, features=tuple(feats))
    fq, cap = bb.run(spec)
    qm = (torch.arange(Lq)[None, :] < lq[:, None])
    q_flat = fq[qm.to(dev)]
    # ---- option rows: own answer tokens only, sorted by length, chunks as wide as their longest option
    lo = torch.tensor([len(t) for t in o_tok], dtype=torch.long)
    M = lo.numel()
    o_flat = torch.empty(int(lo.sum()), fq.shape[-1], dtype=fq.dtype, device=dev)
    o_start = torch.cumsum(lo, 0) - lo
    order = torch.argsort(lo, stable=True)
    q_len_dev = lq.to(torch.int32).to(dev)
    for a in range(0, M, chunk):
        rows = order[a:a + chunk]
        w = max(2, int(lo[rows].max()))
        ids, ln = _rect([o_tok[i] for i in rows.tolist()], bb.pad_id, w)
        rq = row_q[rows]
        pos = (T + lq[rq])[:, None].to(torch.int32) + torch.arange(w, dtype=torch.int32)[None, :]
        spec = PassSpec(ids=ids.to(dev), pos=pos.to(dev), own_hi=ln.to(torch.int32).to(dev), cache=cache,
                        row_state=sidx[rq].to(dev), qkv_prefix=cap, row_q=rq.to(torch.int32).to(dev),
                        q_len=q_len_dev, features=tuple(feats))
        fo, _ = bb.run(spec)
        om = torch.arange(w)[None, :] < ln[:, None]
        # scatter each row's real tokens back to its place in option order
        dst = (o_start[rows][:, None] + torch.arange(w)[None, :])[om]
        o_flat[dst.to(dev)] = fo[om.to(dev)]
    return q_flat, lq, o_flat, lo


def branched_feats(bb: Backbone, tok, questions, cache: KVCache, list_cap: int = 16, chunk: int = 4096):
    """One row [question ; option] per option continuing the state (v3.py:393-444), for calls with few option rows.
    Question features come from each question's first row. Returns (q_flat, lq, o_flat, lo)."""
    dev, feats = bb.device, bb.cfg.feature_layers
    N = len(questions)
    q_tok = tok([answer_row_prefix(q.prompt, q.options, list_cap) for q in questions],
                add_special_tokens=False)["input_ids"]
    o_tok = tok([answer_option_text(o) for q in questions for o in q.options], add_special_tokens=False)["input_ids"]
    n_opt = torch.tensor([len(q.options) for q in questions])
    row_q = torch.repeat_interleave(torch.arange(N), n_opt)
    lq = torch.tensor([len(t) for t in q_tok], dtype=torch.long)
    lo = torch.tensor([len(t) for t in o_tok], dtype=torch.long)
    rows_tok = [q_tok[int(row_q[i])] + o_tok[i] for i in range(len(o_tok))]
    ids, ln = _rect(rows_tok, bb.pad_id)
    W = ids.shape[1]
    sidx = torch.tensor([q.state_idx for q in questions], dtype=torch.int32)
    T = cache.T
    fl = []
    for a in range(0, len(rows_tok), chunk):
        sl = slice(a, a + chunk)
        pos = (T + torch.arange(W, dtype=torch.int32)).expand(ids[sl].shape[0], W)
        spec = PassSpec(ids=ids[sl].to(dev), pos=pos.to(dev), own_hi=ln[sl].to(torch.int32).to(dev), cache=cache,
                        row_state=sidx[row_q[sl]].to(dev), features=tuple(feats))
        fl.append(bb.run(spec)[0])
    Fr = torch.cat(fl, 0)
    first = torch.cumsum(n_opt, 0) - n_opt
    qr, qc, _, _, _ = segment_layout(lq, torch.arange(N), N)
    q_flat = Fr[(first[qr].to(dev), qc.to(dev))]
    r2, c2, _, _, _ = segment_layout(lo, torch.arange(len(o_tok)), len(o_tok))
    o_flat = Fr[(r2.to(dev), (lq[row_q][r2] + c2).to(dev))]
    return q_flat, lq, o_flat, lo


# ------------------------------------------------------------------------------------------------ model
class V3Model:
    """Backbone rows + trunk: run(questions, cache) -> (logits (N, K) fp32, opt_mask (N, K) bool), the
    DecisionModel.run surface (v3.py:588-590) for the branched answer-row configuration.
    question_cache / qcache_min_rows: the serving switch of prepare_inference_ (decider.py:111-116)."""

    def __init__(self, backbone: Backbone, trunk: V3Trunk, tokenizer, list_cap: int = 16,
                 question_cache: bool = True, qcache_min_rows: int = 12, chunk: int = 4096):
        self.backbone, self.trunk, self.tok = backbone, trunk, tokenizer
        self.list_cap, self.question_cache, self.qcache_min_rows, self.chunk = (list_cap, question_cache,
                                                                                qcache_min_rows, chunk)

    def features(self, questions, cache: KVCache):
        if self.question_cache and sum(len(q.options) for q in questions) >= self.qcache_min_rows:
            return branched_feats_qcache(self.backbone, self.tok, questions, cache, self.list_cap, self.chunk)
        return branched_feats(self.backbone, self.tok, questions, cache, self.list_cap, self.chunk)

    def run(self, questions, cache: KVCache):
        dev = self.backbone.device
        n_opt = torch.tensor([len(q.options) for q in questions])
        K = int(n_opt.max())
        opt_mask = (torch.arange(K)[None, :] < n_opt[:, None]).to(dev)
        q_flat, lq, o_flat, lo = self.features(questions, cache)
        state_lens = torch.tensor([cache.lens[q.state_idx] for q in questions], dtype=torch.long)
        logits = self.trunk.forward(q_flat, lq, o_flat, lo, n_opt, opt_mask, state_lens)
        return logits, opt_mask
