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
a softmax layer mix of the multi-layer features. It runs in fp32 on the library's trunk kernels (V3Trunk); its
parameter names are the reference V3's, so a reference checkpoint's trunk loads unchanged.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
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
    lm_feature: bool = False    # v3_lm_feature (v3.py:213-216): the frozen LM's log-prob of each option token


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
    if cfg.lm_feature:                      # drawn last: the other parameters do not depend on the switch
        put("lp_proj", *_lin(g, dm, 1))
        sd["lm_skip"] = torch.tensor(0.3)   # the reference initialises the gate at 0; nonzero exercises the path
    return sd


def trunk_plan(q_lens, o_lens, n_opt, state_lens, up) -> dict:
    """Host-side layout of V3.forward (v3.py:606-662) for the state-free trunk: option-token and question-token
    destinations, option ids and positions, masks; `up` moves each tensor where it is used. q_lens / o_lens /
    n_opt / state_lens are CPU longs (state_lens: the real length of each question's state). The int32 copies and
    the flat destination rows are the kernels' forms of the same layout."""
    N = n_opt.numel()
    K = int(n_opt.max())
    opt_mask = torch.arange(K)[None, :] < n_opt[:, None]
    opt_q = torch.repeat_interleave(torch.arange(N), n_opt)
    opt_k = torch.arange(int(n_opt.sum())) - torch.repeat_interleave(torch.cumsum(n_opt, 0) - n_opt, n_opt)
    row, col, seg, pos, row_len = segment_layout(o_lens, opt_q, N)
    P = int(row_len.max())
    opt_id = torch.full((N, P), -1, dtype=torch.long)
    opt_id[row, col] = opt_k[seg]
    opos = torch.zeros(N, P, dtype=torch.long)
    opos[row, col] = pos
    Tc = int(q_lens.max())
    qrow, qcol, _, _, _ = segment_layout(q_lens, torch.arange(N), N)
    t = torch.arange(Tc)[None, :]
    in_q = t < q_lens[:, None]
    cpos = t + state_lens[:, None]
    c_pad = ~in_q
    return {"N": N, "K": K, "P": P, "Tc": Tc, "rc": (up(row), up(col)), "qrc": (up(qrow), up(qcol)),
            "opt_id": up(opt_id), "opos": up(opos), "in_q": up(in_q), "cpos": up(cpos), "c_pad": up(c_pad),
            "opt_mask": up(opt_mask),
            "rc_flat": up(row * P + col), "qrc_flat": up(qrow * Tc + qcol), "gid32": up(opt_id.int()),
            "cgid32": up(torch.where(c_pad, -1, 0).int()), "opos32": up(opos.int().view(-1)),
            "cpos32": up(cpos.int().view(-1)),
            "olen32": up(row_len.int()), "qlen32": up(q_lens.int()), "nopt32": up(n_opt.int())}


class V3Trunk:
    """The decision trunk on the GPU in fp32 (V3.forward, v3.py:606-709), every op a libod_b200 kernel:
    od_gemm_f32 for every linear (3xTF32 operand pairs on the tensor cores; the projections that read the same input
    stacked into one GEMM: q/k/v of the self-attention, k/v of the cross-attention and of the CLS attention, wg/wv of
    each xATGLU), od_scalenorm_split for each ScaleNorm (with the layer mix for the input projections),
    od_xatglu_split for the xATGLU gate, od_trunk_attn for each attention with its mask from option ids (no
    (N, h, P, P) bias tensor). Residual adds happen in the GEMM epilogues, in place. `params` under the reference
    V3 state-dict names."""

    def __init__(self, cfg: TrunkConfig, params: dict, device):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise _lib.ODError("V3Trunk runs on a CUDA device (libod_b200 has no CPU path)")
        p = {k: v.to(device=self.device, dtype=torch.float32).contiguous() for k, v in params.items()}
        self.p = p

        def w(*names):
            return _lib.split_tf32(torch.cat([p[n + ".weight"] for n in names], 0).contiguous())

        def b(*names):
            return torch.cat([p[n + ".bias"] for n in names], 0).contiguous()

        self.w, self.b = {}, {}
        for n in ("proj_option", "proj_question", "score") + (("rel",) if "rel.weight" in p else ()):
            self.w[n] = w(n)
        blocks = [f"layers.{i}." for i in range(cfg.decision_layers)] + [""]
        for L in blocks:
            ff = L + "ff" if L else "cls_ff"
            self.w[ff + ".wgv"], self.b[ff + ".wgv"] = w(ff + ".wg", ff + ".wv"), b(ff + ".wg", ff + ".wv")
            self.w[ff + ".wo"] = w(ff + ".wo")
        for i in range(cfg.decision_layers):
            L = f"layers.{i}."
            self.w[L + "self_attn.qkv"] = w(L + "self_attn.q", L + "self_attn.k", L + "self_attn.v")
            self.w[L + "self_attn.o"] = w(L + "self_attn.o")
            self.w[L + "cross.q"] = w(L + "cross.q")
            self.w[L + "cross.kv"] = w(L + "cross.k", L + "cross.v")
            self.w[L + "cross.o"] = w(L + "cross.o")
        self.w["cls_attn.q"] = w("cls_attn.q")
        self.w["cls_attn.kv"] = w("cls_attn.k", "cls_attn.v")
        self.w["cls_attn.o"] = w("cls_attn.o")
        self.rope_inv = _lib.rope_table(cfg.d_model // cfg.n_heads, self.device)
        # the layer mix's weights, softmax(layer_mix) as V3._mix_wide (v3.py:328-341) forms them on every call
        self.mix_w = torch.softmax(p["layer_mix"], 0).contiguous() if cfg.n_feat_layers > 1 else None

    def prepare(self, q_lens, o_lens, n_opt, state_lens, up=None) -> dict:
        """trunk_plan uploaded to the trunk's device (once per plan)."""
        return trunk_plan(q_lens, o_lens, n_opt, state_lens, up or (lambda x: x.to(self.device, non_blocking=True)))

    @torch.no_grad()
    def run(self, plan: dict, q_flat: torch.Tensor, o_flat: torch.Tensor, lp_flat: torch.Tensor | None = None,
            want_rel: bool = False):
        """V3.forward's device part (v3.py:627-709): option/context stacks, decision layers, CLS readout, score.
        q_flat (sum lq, nL*d), o_flat (sum lo, nL*d) token features; lp_flat (sum lo,) the LM log-prob of each
        option token (lm_feature). Returns logits (N, K) fp32, NEG at pads; with want_rel also the `rel` head's
        scores of the same final states (v3.py:708), NEG at pads."""
        p, W, B = self.p, self.w, self.b
        L_ = _lib
        h, dm = self.cfg.n_heads, self.cfg.d_model
        N, K, P, Tc = plan["N"], plan["K"], plan["P"], plan["Tc"]
        gid, cgid, opos, cpos = plan["gid32"], plan["cgid32"], plan["opos32"], plan["cpos32"]
        olen, qlen = plan["olen32"], plan["qlen32"]     # real option / question tokens: a prefix of each row
        # The input projections run on the real tokens only and are scattered into the padded (N*P) / (N*Tc) row
        # layouts: ScaleNorm and the projection act row by row, and a padding row (zeros in the reference) projects
        # to the bias alone - proj_option's for option pads, proj_state's for context pads (V3.forward applies
        # proj_state wherever the context is not question text).
        x = p["proj_option.bias"].expand(N * P, dm).contiguous()
        L_.gemm_f32(L_.scalenorm_split(o_flat, p["in_norm.g"], mix_w=self.mix_w), W["proj_option"],
                    bias=p["proj_option.bias"], out=x, out_rows=plan["rc_flat"])
        lpX = None
        if self.cfg.lm_feature:             # token-level log-prob feature (v3.py:666-672): x + lp_proj(lp)
            lpX = torch.zeros(N, P, device=self.device)
            lpX[plan["rc"]] = lp_flat.float()
            x.add_((lpX.view(-1, 1) * p["lp_proj.weight"].view(1, -1)).add_(p["lp_proj.bias"]))
        c = p["proj_state.bias"].expand(N * Tc, dm).contiguous()
        L_.gemm_f32(L_.scalenorm_split(q_flat, p["in_norm.g"], mix_w=self.mix_w), W["proj_question"],
                    bias=p["proj_question.bias"], out=c, out_rows=plan["qrc_flat"])
        for i in range(self.cfg.decision_layers):
            L = f"layers.{i}."
            # x = x + self_attn(n1(x)): RoPE'd within each option, + same_bias[h] between tokens of one option
            qkv = L_.gemm_f32(L_.scalenorm_split(x, p[L + "n1.g"]), W[L + "self_attn.qkv"], rope_pos=opos,
                              rope_inv=self.rope_inv, rope_cols=2 * dm)
            o = L_.trunk_attn(qkv[:, :dm], qkv[:, dm:2 * dm], qkv[:, 2 * dm:], L_.OD_TRUNK_SELF, N, P, P, h,
                              k_grp=gid, q_grp=gid, bonus=p[L + "same_bias"], q_len=olen, k_len=olen)
            L_.gemm_f32(o, W[L + "self_attn.o"], res=x, out=x)
            # x = x + cross(n2(x), n2c(c)): the question tokens, keys RoPE'd at their positions after the state
            qc = L_.gemm_f32(L_.scalenorm_split(x, p[L + "n2.g"]), W[L + "cross.q"])
            kv = L_.gemm_f32(L_.scalenorm_split(c, p[L + "n2c.g"]), W[L + "cross.kv"], rope_pos=cpos,
                             rope_inv=self.rope_inv, rope_cols=dm)
            o = L_.trunk_attn(qc, kv[:, :dm], kv[:, dm:], L_.OD_TRUNK_KEYS, N, P, Tc, h, k_grp=cgid, q_len=olen,
                              k_len=qlen)
            L_.gemm_f32(o, W[L + "cross.o"], res=x, out=x)
            # x = x + ff(n3(x))
            zv = L_.gemm_f32(L_.scalenorm_split(x, p[L + "n3.g"]), W[L + "ff.wgv"], bias=B[L + "ff.wgv"])
            L_.gemm_f32(L_.xatglu_split(zv, p[L + "ff.alpha"]), W[L + "ff.wo"], bias=p[L + "ff.wo.bias"], res=x,
                        out=x)
        # CLS readout: every option's query is the same row (cls.weight, no RoPE); option k sees its own tokens
        qcls = L_.gemm_f32(L_.scalenorm_split(p["cls.weight"], p["cls_nq.g"]), W["cls_attn.q"])
        kv = L_.gemm_f32(L_.scalenorm_split(x, p["cls_nkv.g"]), W["cls_attn.kv"], rope_pos=opos,
                         rope_inv=self.rope_inv, rope_cols=dm)
        o = L_.trunk_attn(qcls, kv[:, :dm], kv[:, dm:], L_.OD_TRUNK_CLS, N, K, P, h, k_grp=gid, q_shared=True,
                          q_len=plan["nopt32"], k_len=olen)
        hc = L_.gemm_f32(o, W["cls_attn.o"], res=p["cls.weight"].view(-1))
        zv = L_.gemm_f32(L_.scalenorm_split(hc, p["cls_nf.g"]), W["cls_ff.wgv"], bias=B["cls_ff.wgv"])
        L_.gemm_f32(L_.xatglu_split(zv, p["cls_ff.alpha"]), W["cls_ff.wo"], bias=p["cls_ff.wo.bias"], res=hc, out=hc)
        hf = L_.scalenorm_split(hc, p["final_norm.g"])
        logits = L_.gemm_f32(hf, W["score"], bias=p["score.bias"]).view(N, K)
        if lpX is not None:                 # gated skip of the length-normalised log-likelihood (v3.py:702-706)
            own_f = (plan["opt_id"][:, None, :] == torch.arange(K, device=self.device)[None, :, None]).float()
            ll = (own_f * lpX[:, None, :]).sum(-1) / own_f.sum(-1).clamp_min(1)
            logits = logits + p["lm_skip"] * ll
        logits = logits.masked_fill(~plan["opt_mask"], NEG)
        if not want_rel:
            return logits
        rel = L_.gemm_f32(hf, W["rel"], bias=p["rel.bias"]).view(N, K).masked_fill(~plan["opt_mask"], NEG)
        return logits, rel


# ------------------------------------------------------------------------------------------------ row plans
def _rect(tok_lists, pad_id, width=None):
    lens = torch.tensor([len(t) for t in tok_lists], dtype=torch.long)
    L = width or max(1, int(lens.max()))
    ids = torch.full((len(tok_lists), L), pad_id, dtype=torch.long)
    for i, t in enumerate(tok_lists):
        ids[i, : len(t)] = torch.tensor(t, dtype=torch.long)
    return ids, lens


@dataclass
class RowPass:
    """One rectangular backbone pass over option (or question) rows, with the scatter of its real tokens."""
    spec: PassSpec
    dst: torch.Tensor | None = None     # destination index of each real token in the flat feature array
    keep: torch.Tensor | None = None    # flat (row * w + token) indices of the pass's real tokens, int64: gathering
                                        # by index needs no device-to-host read, unlike a boolean mask


@dataclass
class RowPlan:
    """Everything the row passes of one call need, built on the host and uploaded once (no host sync later)."""
    qcache: bool
    question: RowPass | None            # question pass (question cache) with the flat question-token mask
    options: list                       # RowPass per option chunk (or per [question ; option] chunk)
    n_q_tok: int
    n_o_tok: int
    q_lens: torch.Tensor                # CPU
    o_lens: torch.Tensor                # CPU
    q_src: tuple | None = None          # rows-path: (row, col) of question tokens in the first row of each question
    lp_osrc: torch.Tensor | None = None # lm_feature: per option token, the o_flat row of the previous token ...
    lp_first: torch.Tensor | None = None  # ... except an option's first token (these positions of the flat array)
    lp_qsrc: torch.Tensor | None = None # ... which takes its question's last token from q_flat
    lp_tok: torch.Tensor | None = None  # the option tokens (targets), int64


def _flat_idx(mask: torch.Tensor) -> torch.Tensor:
    """Flat indices of the True entries of a host mask (computed at plan time)."""
    return torch.nonzero(mask.reshape(-1)).view(-1)


def width_chunks(lengths: torch.Tensor, chunk: int, waste: float = 0.25) -> list:
    """Split rows sorted by length (ascending) into chunks: a new chunk starts when it would exceed `chunk` tokens
    (rows x its width) or when padding the chunk to a longer row would waste more than `waste` of its tokens.
    Returns [(start, end)] over the sorted rows."""
    out, a, w = [], 0, 0
    for i, L in enumerate(lengths.tolist()):
        n = i - a
        if n and ((n + 1) * max(w, L, 2) > chunk or (L > w and (L - w) * n > waste * n * w)):
            out.append((a, i))
            a, n, w = i, 0, 0
        w = max(w, L)
    if a < lengths.numel():
        out.append((a, lengths.numel()))
    return out


def row_groups(owner: torch.Tensor, max_rows: int) -> torch.Tensor:
    """(G, 2) [first row, rows] runs of consecutive rows with the same owner (question), at most max_rows each."""
    groups, a = [], 0
    o = owner.tolist()
    for i in range(1, len(o) + 1):
        if i == len(o) or o[i] != o[a] or i - a == max_rows:
            groups.append((a, i - a))
            a = i
    return torch.tensor(groups, dtype=torch.int32).view(-1, 2)


def lm_sources(q_tok, o_tok, lq, lo, row_q, up) -> dict:
    """Where each option token's LM log-prob reads its previous position (v3.py:437-442, 527-532): the option's
    previous token in o_flat, or for its first token its question's last token in q_flat; and the targets."""
    q_start = torch.cumsum(lq, 0) - lq
    o_start = torch.cumsum(lo, 0) - lo
    n = int(lo.sum())
    m_of = torch.repeat_interleave(torch.arange(lo.numel()), lo)
    first = torch.arange(n) == o_start[m_of]
    osrc = (torch.arange(n) - 1).clamp_min(0)
    qm = row_q[m_of[first]]
    targets = torch.tensor([t for ts in o_tok for t in ts], dtype=torch.long)
    return {"lp_osrc": up(osrc), "lp_first": up(torch.nonzero(first).view(-1)),
            "lp_qsrc": up(q_start[qm] + lq[qm] - 1), "lp_tok": up(targets)}


def plan_rows(bb: Backbone, tok, questions, T: int, qcache: bool, list_cap: int = 16, chunk: int = 1 << 18,
              up=None, lm: bool = False) -> RowPlan:
    """Host layout of the branched row passes. qcache: V3._branched_feats_qcache (v3.py:446-534) - one right-padded
    question pass continuing each question's state at positions T + j, capturing its K/V, then option rows of
    their own answer tokens (sorted by length, chunks as wide as their longest option, positions after their own
    question). Otherwise V3._branched_feats (v3.py:393-444) - one row [question ; option] per option. chunk: the most
    tokens one row pass holds (its activations; fewer passes re-read the cached state less often)."""
    dev = bb.device
    up = up or (lambda x: x.to(dev, non_blocking=True))
    N = len(questions)
    q_tok = tok([answer_row_prefix(q.prompt, q.options, list_cap) for q in questions],
                add_special_tokens=False)["input_ids"]
    o_tok = tok([answer_option_text(o) for q in questions for o in q.options], add_special_tokens=False)["input_ids"]
    n_opt = torch.tensor([len(q.options) for q in questions])
    row_q = torch.repeat_interleave(torch.arange(N), n_opt)
    sidx = torch.tensor([q.state_idx for q in questions], dtype=torch.int32)
    lq = torch.tensor([len(t) for t in q_tok], dtype=torch.long)
    lo = torch.tensor([len(t) for t in o_tok], dtype=torch.long)
    feats = tuple(bb.cfg.feature_layers)
    M = lo.numel()
    if qcache:
        Qids, _ = _rect(q_tok, bb.pad_id)
        Lq = Qids.shape[1]
        qpos = (T + torch.arange(Lq, dtype=torch.int32)).expand(N, Lq).contiguous()
        qkeep = torch.arange(Lq)[None, :] < lq[:, None]
        qpass = RowPass(PassSpec(ids=up(Qids), pos=up(qpos), own_hi=up(lq.to(torch.int32)), row_state=up(sidx),
                                 capture=True, features=feats), keep=up(_flat_idx(qkeep)))
        o_start = torch.cumsum(lo, 0) - lo
        order = torch.argsort(lo, stable=True)
        q_len_dev = up(lq.to(torch.int32))
        passes = []
        rep = bb.cfg.heads // bb.cfg.kv_heads
        for a, b in width_chunks(lo[order], chunk):
            rows = order[a:b]
            w = max(2, int(lo[rows].max()))
            ids, ln = _rect([o_tok[i] for i in rows.tolist()], bb.pad_id, w)
            rq = row_q[rows]
            pos = (T + lq[rq])[:, None].to(torch.int32) + torch.arange(w, dtype=torch.int32)[None, :]
            keep = torch.arange(w)[None, :] < ln[:, None]
            dst = (o_start[rows][:, None] + torch.arange(w)[None, :])[keep]
            # rows of one question (consecutive after the stable length sort) share a tensor-core tile
            mg = max(1, _lib.ATTN_CTA_SLOTS // (w * rep))
            grp = row_groups(rq, mg)
            passes.append(RowPass(PassSpec(ids=up(ids), pos=up(pos), own_hi=up(ln.to(torch.int32)),
                                           row_state=up(sidx[rq]), row_q=up(rq.to(torch.int32)), q_len=q_len_dev,
                                           row_groups=up(grp), max_group_rows=int(grp[:, 1].max()),
                                           features=feats), dst=up(dst), keep=up(_flat_idx(keep))))
        return RowPlan(True, qpass, passes, int(lq.sum()), int(lo.sum()), lq, lo,
                       **(lm_sources(q_tok, o_tok, lq, lo, row_q, up) if lm else {}))
    rows_tok = [q_tok[int(row_q[i])] + o_tok[i] for i in range(M)]
    ids, ln = _rect(rows_tok, bb.pad_id)
    W = ids.shape[1]
    passes = []
    o_dst_start = torch.cumsum(lo, 0) - lo
    rows_per = max(1, chunk // max(1, W))
    for a in range(0, M, rows_per):
        sl = slice(a, min(a + rows_per, M))
        R = sl.stop - sl.start
        pos = (T + torch.arange(W, dtype=torch.int32)).expand(R, W).contiguous()
        # option tokens of these rows: columns [lq, lq + lo) of each row
        rr = torch.arange(sl.start, sl.stop)
        cols = torch.arange(W)[None, :]
        keep = (cols >= lq[row_q[rr]][:, None]) & (cols < (lq[row_q[rr]] + lo[rr])[:, None])
        dst = (o_dst_start[rr][:, None] + cols - lq[row_q[rr]][:, None])[keep]
        passes.append(RowPass(PassSpec(ids=up(ids[sl]), pos=up(pos), own_hi=up(ln[sl].to(torch.int32)),
                                       row_state=up(sidx[row_q[sl]]), features=feats), dst=up(dst),
                              keep=up(_flat_idx(keep))))
    first = torch.cumsum(n_opt, 0) - n_opt
    qr, qc, _, _, _ = segment_layout(lq, torch.arange(N), N)
    return RowPlan(False, None, passes, int(lq.sum()), int(lo.sum()), lq, lo, (up(first[qr]), up(qc)),
                   **(lm_sources(q_tok, o_tok, lq, lo, row_q, up) if lm else {}))


def run_rows(bb: Backbone, plan: RowPlan, cache: KVCache):
    """Device part of the row passes. Returns (q_flat, o_flat) features (tokens, nL*H) bf16."""
    dev = bb.device
    nf = len(bb.cfg.feature_layers) * bb.cfg.hidden
    o_flat = torch.empty(plan.n_o_tok, nf, dtype=bb.cfg.dtype, device=dev)
    if plan.qcache:
        qspec = plan.question.spec
        qspec.cache = cache
        fq, cap = bb.run(qspec)
        q_flat = fq.view(-1, fq.shape[-1])[plan.question.keep]
        for rp in plan.options:
            rp.spec.cache, rp.spec.qkv_prefix = cache, cap
            fo, _ = bb.run(rp.spec)
            o_flat[rp.dst] = fo.view(-1, fo.shape[-1])[rp.keep]
        return q_flat, o_flat
    q_flat = None
    first_rows = []
    for rp in plan.options:
        rp.spec.cache = cache
        fo, _ = bb.run(rp.spec)
        o_flat[rp.dst] = fo.view(-1, fo.shape[-1])[rp.keep]
        first_rows.append(fo)
    Fr = torch.cat(first_rows, 0) if len(first_rows) > 1 else first_rows[0]
    q_flat = Fr[plan.q_src]
    return q_flat, o_flat


# ------------------------------------------------------------------------------------------------ model
class V3Model:
    """Backbone rows + trunk, the DecisionModel.run surface (v3.py:588-590) for the branched answer-row
    configuration. question_cache / qcache_min_rows: the serving switch of prepare_inference_ (decider.py:111-116)."""

    def __init__(self, backbone: Backbone, trunk: V3Trunk, tokenizer, list_cap: int = 16,
                 question_cache: bool = True, qcache_min_rows: int = 12, chunk: int = 1 << 18):
        self.backbone, self.trunk, self.tok = backbone, trunk, tokenizer
        self.list_cap, self.question_cache, self.qcache_min_rows, self.chunk = (list_cap, question_cache,
                                                                                qcache_min_rows, chunk)

    def plan(self, questions, T: int, state_lens: list, up=None):
        qc = self.question_cache and sum(len(q.options) for q in questions) >= self.qcache_min_rows
        rows = plan_rows(self.backbone, self.tok, questions, T, qc, self.list_cap, self.chunk, up,
                         lm=self.trunk.cfg.lm_feature)
        n_opt = torch.tensor([len(q.options) for q in questions])
        sl = torch.tensor([state_lens[q.state_idx] for q in questions], dtype=torch.long)
        return rows, self.trunk.prepare(rows.q_lens, rows.o_lens, n_opt, sl, up)

    def execute(self, plan, cache: KVCache):
        rows, tplan = plan
        q_flat, o_flat = run_rows(self.backbone, rows, cache)
        lp = None
        if self.trunk.cfg.lm_feature:
            # the final normed hidden state (the last feature layer) of the position before each option token
            bb = self.backbone
            assert bb.cfg.feature_layers[-1] == "final", "the LM feature reads the 'final' feature layer"
            H = bb.cfg.hidden
            h_prev = o_flat[rows.lp_osrc, -H:]
            h_prev[rows.lp_first] = q_flat[rows.lp_qsrc, -H:]
            lp = bb.token_logprob(h_prev.contiguous(), rows.lp_tok)
        return self.trunk.run(tplan, q_flat, o_flat, lp), tplan["opt_mask"]

    def run(self, questions, cache: KVCache):
        """(logits (N, K) fp32, opt_mask (N, K) bool) for questions reading `cache`."""
        return self.execute(self.plan(questions, cache.T, cache.lens), cache)
