"""CPU oracle of the whole decision forward pass - TEST INFRASTRUCTURE and the timed CPU baseline, never the product.

A PyTorch-CPU restatement of the reference's path with its bf16 rounding points (what src/opendecider computes with
the transformers Qwen3.5 modules on a bf16 CPU model):
  decoder        Qwen3_5DecoderLayer / Qwen3_5Attention / Qwen3_5MLP / Qwen3_5RMSNorm
                 (transformers models/qwen3_5/modeling_qwen3_5.py:620-783), every linear through the A8W8 arithmetic
                 installed at the reference's Int8Linear._fused seam (quant.py:150-152): per-token int8 activations by
                 Int8Tensor.quantize's formula (quant.py:37-41, fp32 scale), exact int32 products (torch._int_mm),
                 bf16((acc * s_x) * s_w); weights quantised as Int8Linear does (quant.py:124-127)
  state pass     Backbone.prefix_cache_batch (backbone.py:347-368): left-padded, causal, the cache quantised per
                 (state, head, token) by Int8Tensor.quantize (backbone.py:446)
  row passes     V3._branched_feats_qcache (v3.py:446-534): one right-padded question pass over every question, then
                 option rows sorted by length in chunks of 64; each attention call routed as shared_prefix_attention
                 routes it (prefix_attn.py:135-175): one masked scaled_dot_product_attention call for rows of several
                 states (prefix_attn.py:102-117), else _split_attention's CPU branch per state (prefix_attn.py:58-76)
  attention      the reference's own CPU calls: torch's scaled_dot_product_attention (its flash kernel on the CPU) for
                 the state pass and the one-call path, so the oracle equals the reference bit for bit end to end
  trunk/readout  oracle/trunk.py's fp32 restatement of the V3 trunk (pinned to the reference by
                 tests/golden/e2e_config1.npz) and Decider._probs' softmax (decider.py:255-257)
Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline, --impl reference) may import this module.
"""
from __future__ import annotations

import torch

from . import ops

BF = torch.bfloat16


def _quant_w(w: torch.Tensor):
    wf = w.float()
    s = wf.abs().amax(1, keepdim=True).clamp_min(1e-8) / 127.0
    return torch.round(wf / s).clamp_(-127, 127).to(torch.int8), s.to(w.dtype)


def a8w8(x: torch.Tensor, qw: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """bf16 x (M, K) through the W8A8 arithmetic; qw (N, K) int8, sw (N, 1) bf16 -> bf16 (M, N)."""
    xf = x.float()
    s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 127.0
    q = torch.round(xf / s).clamp_(-127, 127).to(torch.int8)
    M = q.shape[0]
    if M <= 16:                                                 # _int_mm wants more than 16 rows: zero rows are exact
        q = torch.cat([q, q.new_zeros(17 - M, q.shape[1])])
    acc = torch._int_mm(q, qw.t())[:M]
    return ((acc.float() * s) * sw.float().view(1, -1)).to(BF)


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (out * (1.0 + w.float())).to(x.dtype)


def _rot(x, cos, sin):
    D = x.shape[-1]
    rh = torch.cat([-x[..., D // 2:], x[..., : D // 2]], -1)
    return (x * cos) + (rh * sin)


class OracleDecoder:
    """The int8 decoder on the CPU. sd: float (bf16) weights under HF's Qwen3_5TextModel names; `layers` limits the
    pass to the first n layers (the timed baseline samples a few layers and extrapolates). smooth: SmoothQuant scales
    s (K,) per linear keyed relative to the layer list ('{i}.self_attn.q_proj', as the reference's scale files are):
    smooth_a8w8_ (quant.py:333-350) stores W * s (fp32 product, weight dtype) and SmoothedLinear.forward
    (quant.py:328-329) multiplies the input by inv_s = bf16(1 / s) in the activation dtype before the A8W8 product."""

    def __init__(self, cfg, sd: dict, layers: int | None = None, smooth: dict | None = None):
        self.cfg = cfg
        self.n = layers or cfg.layers
        self.q, self.inv = {}, {}
        smooth = smooth or {}
        for name, w in sd.items():
            if not name.endswith("norm.weight"):
                base = name[: -len(".weight")]
                sv = smooth.get(base[len("layers."):]) if base.startswith("layers.") else None
                if sv is not None:
                    sv = sv.float()
                    w = (w.float() * sv[None, :]).to(w.dtype)
                    self.inv[base] = (1.0 / sv).to(BF)
                self.q[base] = _quant_w(w)
        self.norm = {k: v for k, v in sd.items() if k.endswith("norm.weight")}
        self.cos, self.sin = ops.rope_tables(cfg.head_dim, cfg.rope_theta, cfg.max_pos)

    def lin(self, name: str, x: torch.Tensor) -> torch.Tensor:
        """One projection: [SmoothedLinear's bf16(x * inv_s)] then the A8W8 arithmetic. x (M, K) bf16."""
        inv = self.inv.get(name)
        if inv is not None:
            x = x * inv
        return a8w8(x, *self.q[name])

    def embed(self, ids):
        qw, s = self.q["embed_tokens"]
        return qw[ids].to(BF) * s[ids]

    def layer(self, i, x, pos, attend):
        """One decoder layer on (R, t, H) bf16; attend(i, q, k, v) -> (R, t, Hq*D) bf16. Returns (x, k, v)."""
        cfg, p = self.cfg, f"layers.{i}."
        R, t, H = x.shape
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        h = rmsnorm(x, self.norm[p + "input_layernorm.weight"], cfg.eps).reshape(R * t, H)
        qg = self.lin(p + "self_attn.q_proj", h).view(R, t, Hq, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(R, t, Hq * D)
        k = self.lin(p + "self_attn.k_proj", h).view(R, t, Hkv, D)
        v = self.lin(p + "self_attn.v_proj", h).view(R, t, Hkv, D)
        q = rmsnorm(q, self.norm[p + "self_attn.q_norm.weight"], cfg.eps)
        k = rmsnorm(k, self.norm[p + "self_attn.k_norm.weight"], cfg.eps)
        c, s = self.cos[pos][:, :, None, :], self.sin[pos][:, :, None, :]
        q, k = _rot(q, c, s), _rot(k, c, s)
        o = attend(i, q, k, v) * torch.sigmoid(gate)
        x = x + self.lin(p + "self_attn.o_proj", o.reshape(R * t, Hq * D)).view(R, t, H)
        h2 = rmsnorm(x, self.norm[p + "post_attention_layernorm.weight"], cfg.eps).reshape(R * t, H)
        g = self.lin(p + "mlp.gate_proj", h2)
        u = self.lin(p + "mlp.up_proj", h2)
        m = torch.nn.functional.silu(g) * u
        x = x + self.lin(p + "mlp.down_proj", m).view(R, t, H)
        return x, k, v

    def run(self, ids, pos, attend, features=()):
        """Rows (R, t) -> per-layer (k, v) and the requested features (R, t, nL*H) bf16."""
        x = self.embed(ids)
        feats, kv = {}, []
        for i in range(self.n):
            x, k, v = self.layer(i, x, pos, attend)
            kv.append((k, v))
            feats[i + 1] = x
        out = None
        if features:
            feats["final"] = rmsnorm(x, self.norm["norm.weight"], self.cfg.eps)
            out = torch.cat([feats[f if f == "final" else int(f)] for f in features], -1)
        return out, kv


def sdpa_flash(q, k, v, ok):
    """The attention of every batched pass the reference runs through torch's scaled_dot_product_attention with a
    boolean mask - the transformers sdpa interface of its state pass (modeling_qwen3_5.py:676-686 ->
    integrations/sdpa_attention.py) and shared_prefix_attention's one-call multi-state path (prefix_attn.py:102-117).
    On the CPU that call runs torch's flash-attention kernel (fp32 scores, probabilities rounded to bf16 before the
    P.V product, key blocks of 512 with running-max rescaling); the oracle makes the same call on the CPU, so its
    arithmetic is the reference's own, bit for bit. Query rows with no visible key attend every key instead, as
    transformers' sdpa mask does for them (their outputs feed no real token). q (R, t, Hq, D), k/v (R, Tk, Hkv, D)
    bf16, ok (R, t, Tk) bool -> (R, t, Hq*D) bf16."""
    R, t, Hq, D = q.shape
    g = Hq // k.shape[2]
    ok = ok | ~ok.any(-1, keepdim=True)
    qq = q.transpose(1, 2)
    kk = k.repeat_interleave(g, 2).transpose(1, 2)
    vv = v.repeat_interleave(g, 2).transpose(1, 2)
    o = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=ok[:, None], scale=D ** -0.5)
    return o.transpose(1, 2).reshape(R, t, Hq * D)


def causal_attend(pad, sdpa=None):
    """Causal attention of the state pass with left padding (keys before pad[r] masked)."""
    def f(i, q, k, v):
        t = q.shape[1]
        j = torch.arange(t)
        ok = (j[None, :] <= j[:, None])[None] & (j[None, None, :] >= pad.view(-1, 1, 1))
        return (sdpa or sdpa_flash)(q, k, v, ok)
    return f


def sdpa_exp_variant(q, k, v, ok):
    """sdpa_flash with ONE change, for measuring how sensitive a decision is to the last bit of attention: torch.exp
    in place of the CPU flash kernel's own vectorised exponential and a division in place of its reciprocal
    multiply. Scores, masks, the bf16 rounding of the probabilities and the fp32 accumulation are unchanged; about 9 %
    of the bf16 outputs move by one ulp. Any attention not bit-identical to torch's CPU kernel (a tensor-core kernel
    with its own exponential and summation order) differs from the reference by perturbations of this size."""
    R, t, Hq, D = q.shape
    g = Hq // k.shape[2]
    ok = ok | ~ok.any(-1, keepdim=True)
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(g, 2).transpose(1, 2)
    vf = v.float().repeat_interleave(g, 2).transpose(1, 2)
    s = ((qf @ kf.transpose(-1, -2)) * D ** -0.5).masked_fill(~ok[:, None], float("-inf"))
    p = torch.exp(s - s.amax(-1, keepdim=True))
    o = (p.to(BF).float() @ vf) / p.sum(-1, keepdim=True)
    return o.transpose(1, 2).reshape(R, t, Hq * D).to(BF)


BATCHED_BYTES = 1 << 30     # prefix_attn.py:27: the one-call multi-state path's bound on gathered prefix K/V


def uses_batched_call(n_rows: int, n_states: int, hkv: int, d: int, prefix_len: int) -> bool:
    """shared_prefix_attention's choice (prefix_attn.py:159-167): rows reading more than one state go through ONE
    masked scaled_dot_product_attention call per layer when rows x (Hkv * D * prefix length) bf16 values x 4 stays
    within BATCHED_BYTES; otherwise (and always for a single state) through _split_attention, one state at a time."""
    return n_states > 1 and n_rows * hkv * d * prefix_len * 2 * 4 <= BATCHED_BYTES


def split_rows(q, k, v, Kp, Vp, pm):
    """_forward's per-state branch (prefix_attn.py:118-129) for rows of one state: the prefix from its first real key
    (leading pads sliced off), later pads masked, then _split_attention's CPU branch (fp32 throughout).
    q (n, t, Hq, D), k/v (n, t, Hkv, D), Kp/Vp (Hkv, P, D), pm (P,) bool -> (n, t, Hq*D) bf16."""
    n, t, Hq, D = q.shape
    off = int(pm.int().argmax())
    holes = bool((~pm).sum() > off)
    o = ops.split_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), Kp[:, off:], Vp[:, off:],
                            pm[off:] if holes else None, D ** -0.5)
    return o.to(BF).transpose(1, 2).reshape(n, t, Hq * D)


class OracleDecision:
    """decide_many on the CPU: state pass, question-cache row passes, trunk, readout."""

    def __init__(self, cfg, sd, trunk, tok, temps: dict, temperature: float, layers: int | None = None,
                 list_cap: int = 16, qcache_min_rows: int = 12, none_text: str = "none of the above",
                 branch_chunk: int = 64, sdpa=None, smooth: dict | None = None):
        self.dec = OracleDecoder(cfg, sd, layers, smooth)
        self.cfg, self.trunk, self.tok, self.temps, self.temperature = cfg, trunk, tok, temps, temperature
        self.list_cap, self.qcache_min_rows, self.none_text = list_cap, qcache_min_rows, none_text
        self.branch_chunk = branch_chunk                  # v3_branch_chunk (models.py:66)
        self.sdpa = sdpa or sdpa_flash                    # sdpa_exp_variant: the sensitivity probe

    def state_pass(self, states):
        from opendecider_b200.batching import state_text
        seqs = self.tok([state_text(s) for s in states], add_special_tokens=False)["input_ids"]
        lens = [len(s) for s in seqs]
        S, T = len(seqs), max(lens)
        ids = torch.tensor([[0] * (T - n) + list(s) for s, n in zip(seqs, lens)])
        pad = torch.tensor([T - n for n in lens])
        pos = torch.arange(T).expand(S, T)
        _, kv = self.dec.run(ids, pos, causal_attend(pad, self.sdpa))
        cache = []
        for k, v in kv:                                   # Int8Tensor.quantize then materialize(): bf16 prefix
            kq, ks, _ = ops.quantize_rows(k.transpose(1, 2).float().numpy(), "bf16")
            vq, vs, _ = ops.quantize_rows(v.transpose(1, 2).float().numpy(), "bf16")
            cache.append((ops.materialize_int8(torch.from_numpy(kq), torch.from_numpy(ks).to(BF)),
                          ops.materialize_int8(torch.from_numpy(vq), torch.from_numpy(vs).to(BF))))
        return cache, pad, T, lens

    def append_pass(self, prebuilt, appends):
        """PrefixCache.encode's continuation of cached states (state_cache.py:116-158, one request at a time there):
        the appended ids (equal counts) attend the materialised prefix and each other causally at positions T..T+n-1
        (Backbone.prefill with the restored cache); their K/V are quantised into the next snapshot (_take,
        state_cache.py:79); PackedCache.pack then quantises the whole cache (the materialised prefix again, and the
        new K/V) and the rows read it materialised. Returns ((cache, pad, T + n, lens + n), snapshots, packs) with
        snapshots[layer] = ((k int8 (S, Hkv, n, D), k scale bf16 (S, Hkv, n)), (v ...)) and packs[layer] the same
        over all T + n tokens."""
        cache, pad, T, lens = prebuilt
        seqs = self.tok(list(appends), add_special_tokens=False)["input_ids"]
        S, n = len(seqs), len(seqs[0])
        assert all(len(q) == n for q in seqs)
        ids = torch.tensor(seqs)
        pos = (T + torch.arange(n)).expand(S, n)
        pm_state = torch.arange(T)[None, :] >= pad[:, None]
        D = self.cfg.head_dim

        i_ = torch.arange(n)
        ok = torch.cat([pm_state[:, None, :].expand(S, n, T), (i_[None, :] <= i_[:, None])[None].expand(S, n, n)], 2)

        def attend(i, q, k, v):
            Kp, Vp = cache[i]                                             # (S, Hkv, T, D) materialised
            return self.sdpa(q, torch.cat([Kp.transpose(1, 2), k], 1), torch.cat([Vp.transpose(1, 2), v], 1), ok)

        _, kv = self.dec.run(ids, pos, attend)
        new, snaps, packs = [], [], []
        for (Kp, Vp), (k, v) in zip(cache, kv):
            pair, snap, pack = [], [], []
            for P_, x in ((Kp, k), (Vp, v)):
                xn = x.transpose(1, 2).contiguous()                       # (S, Hkv, n, D) bf16
                q8, sc, _ = ops.quantize_rows(xn.float().numpy(), "bf16")
                snap.append((torch.from_numpy(q8), torch.from_numpy(sc).to(BF).reshape(q8.shape[:-1])))
                full = torch.cat([P_, xn], 2)
                fq, fs, _ = ops.quantize_rows(full.float().numpy(), "bf16")
                fq, fs = torch.from_numpy(fq), torch.from_numpy(fs).to(BF).reshape(fq.shape[:-1])
                pack.append((fq, fs))
                pair.append(ops.materialize_int8(fq, fs[..., None]))
            new.append(tuple(pair))
            snaps.append(tuple(snap))
            packs.append(tuple(pack))
        return (new, pad, T + n, [l + n for l in lens]), snaps, packs

    def decide(self, requests, prebuilt=None):
        """Returns (probs (N, K), renorm (N, K) fp64, p_none (N,)) numpy, questions in request order. prebuilt: the
        states' (cache, pad, T, lens) from state_pass / append_pass instead of a state pass."""
        import copy
        from opendecider_b200.batching import MAX_OPTIONS, answer_option_text, answer_row_prefix
        cache, pad, T, lens = prebuilt if prebuilt is not None else self.state_pass([r.state for r in requests])
        qs = []
        for i, r in enumerate(requests):
            for q in r.questions:
                q2 = copy.copy(q)
                q2.state_idx = i
                if len(q.options) < MAX_OPTIONS:
                    q2.options = list(q.options) + [self.none_text]
                    q2.none_col = len(q.options)
                qs.append(q2)
        N = len(qs)
        q_tok = self.tok([answer_row_prefix(q.prompt, q.options, self.list_cap) for q in qs])["input_ids"]
        o_tok = self.tok([answer_option_text(o) for q in qs for o in q.options])["input_ids"]
        n_opt = torch.tensor([len(q.options) for q in qs])
        row_q = torch.repeat_interleave(torch.arange(N), n_opt)
        lq = torch.tensor([len(t) for t in q_tok])
        lo = torch.tensor([len(t) for t in o_tok])
        sidx = torch.tensor([q.state_idx for q in qs])
        feats = tuple(self.cfg.feature_layers)
        Lq = int(lq.max())
        Qids = torch.zeros(N, Lq, dtype=torch.long)
        for j, t in enumerate(q_tok):
            Qids[j, : len(t)] = torch.tensor(t)
        pm_state = torch.arange(T)[None, :] >= pad[:, None]
        Hkv, D = self.cfg.kv_heads, self.cfg.head_dim
        qmask = torch.arange(Lq)[None, :] < lq[:, None]
        causal = lambda t: torch.arange(t)[None, :] <= torch.arange(t)[:, None]

        # the question pass: ONE right-padded pass over every question (v3_question_batch, v3.py:484-499), reading
        # the state prefix through shared_prefix_attention (one masked call, or one state at a time)
        batched_q = uses_batched_call(N, len(set(sidx.tolist())), Hkv, D, T)

        def attend_q(i, q, k, v):
            Kp, Vp = cache[i]                                             # (S, Hkv, T, D) materialised
            if batched_q:
                ok = torch.cat([pm_state[sidx][:, None, :].expand(N, Lq, T), causal(Lq)[None].expand(N, Lq, Lq)], 2)
                return self.sdpa(q, torch.cat([Kp[sidx].transpose(1, 2), k], 1),
                                  torch.cat([Vp[sidx].transpose(1, 2), v], 1), ok)
            out = torch.empty(N, Lq, q.shape[2] * D, dtype=BF)
            for st in sorted(set(sidx.tolist())):
                r = (sidx == st).nonzero().squeeze(1)
                out[r] = split_rows(q[r], k[r], v[r], Kp[st], Vp[st], pm_state[st])
            return out

        qpos = (T + torch.arange(Lq)).expand(N, Lq)
        fq, qkv = self.dec.run(Qids, qpos, attend_q, feats)
        q_flat = fq[qmask]
        o_flat = torch.empty(int(lo.sum()), fq.shape[-1], dtype=fq.dtype)
        o_start = torch.cumsum(lo, 0) - lo
        # option rows (v3.py:500-519): every question's rows sorted by option length (stable), chunks of
        # v3_branch_chunk rows, each as wide as its longest option (>= 2), right-padded; a row's tokens continue at its
        # own question's end; the prefix is [state ; question] (pmq masks both levels' pads)
        pmq = torch.cat([pm_state[sidx], qmask], 1)                       # (N, T + Lq)
        order = torch.argsort(lo, stable=True)
        for a in range(0, order.numel(), self.branch_chunk):
            rs = order[a: a + self.branch_chunk]
            n, w = rs.numel(), max(2, int(lo[rs].max()))
            ids = torch.zeros(n, w, dtype=torch.long)
            for j, m in enumerate(rs.tolist()):
                ids[j, : lo[m]] = torch.tensor(o_tok[m])
            qr = row_q[rs]
            batched = uses_batched_call(n, len(set(qr.tolist())), Hkv, D, T + Lq)

            def attend_o(i, q, k, v, qr=qr, batched=batched):
                Kp, Vp = cache[i]
                Kq, Vq = qkv[i]                                           # (N, Lq, Hkv, D) captured
                Kc = torch.cat([Kp[sidx].transpose(1, 2), Kq], 1)         # (N, T + Lq, Hkv, D)
                Vc = torch.cat([Vp[sidx].transpose(1, 2), Vq], 1)
                if batched:
                    t = q.shape[1]
                    ok = torch.cat([pmq[qr][:, None, :].expand(len(qr), t, T + Lq),
                                    causal(t)[None].expand(len(qr), t, t)], 2)
                    return self.sdpa(q, torch.cat([Kc[qr], k], 1), torch.cat([Vc[qr], v], 1), ok)
                qj = int(qr[0])
                return split_rows(q, k, v, Kc[qj].transpose(0, 1), Vc[qj].transpose(0, 1), pmq[qj])

            pos = (T + lq[qr])[:, None] + torch.arange(w)[None, :]
            fo, _ = self.dec.run(ids, pos, attend_o, feats)
            for j, m in enumerate(rs.tolist()):
                o_flat[o_start[m]: o_start[m] + lo[m]] = fo[j, : lo[m]]
        sl = torch.tensor([lens[q.state_idx] for q in qs])
        tplan = self.trunk.prepare(lq, lo, n_opt, sl)
        lp = None
        if self.trunk.cfg.lm_feature:
            # V3's LM feature (v3.py:527-532): each option token's log-prob given the final normed hidden state of
            # the position before it - the previous option token, or for the first its question's last token
            H = self.cfg.hidden
            q_start = torch.cumsum(lq, 0) - lq
            rows_prev = []
            for m in range(lo.numel()):
                qj = int(row_q[m])
                rows_prev.append(q_flat[int(q_start[qj] + lq[qj] - 1), -H:])
                for c in range(1, int(lo[m])):
                    rows_prev.append(o_flat[int(o_start[m]) + c - 1, -H:])
            h_prev = torch.stack(rows_prev)
            tgt = torch.tensor([t for ts in o_tok for t in ts], dtype=torch.long)
            qw, sw = self.dec.q["embed_tokens"]
            lp = ops.token_logprob(h_prev, qw, sw, tgt)
        logits = self.trunk.run(tplan, q_flat, o_flat, lp)
        Tq = [self.temps.get(q.type, self.temperature) for q in qs]
        nc = [getattr(q, "none_col", -1) for q in qs]
        probs, ren, pn = ops.readout(logits.numpy(), Tq, tplan["opt_mask"].numpy(), none_col=nc)
        return probs, ren, pn, logits
