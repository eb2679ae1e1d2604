"""Drop-in installation of the B200 kernels into the reference's own model (src/opendecider), at the seams the
reference itself defines, next to its prepare_inference_ (decider.py:91-117):

  GEMM seam        every int8 linear of the backbone (the reference's Int8Linear, also inside a SmoothedLinear) gets
                   a W8A8 callable in its `_fused` slot (Int8Linear.forward, quant.py:149-152) - the slot
                   int8_to_gemlite_ fills (quant.py:398-409). The modules stay in the tree, so forward hooks on them
                   (VeRA, vera.py:54) keep firing on their outputs.
  attention seam   the reference's shared_prefix_attention (prefix_attn.py:135-175) is replaced, in the module that
                   calls it (opendecider.v3), by b200_shared_prefix_attention: same signature and the same per-layer
                   forward swap, but attention reads the PackedCache's Int8Tensor K/V directly in od_prefix_attn (the
                   int8 prefix dequantised in the kernel, the question level of the question cache as a second
                   prefix, the row's own keys causally) - no materialize() of the state K/V (prefix_attn.py:146-149),
                   no per-state loop, no host synchronisation.
  trunk seam       a V3 model in the serving configuration (branched answer rows, question cross-attention, readout
                   "last") gets b200_v3_forward in place of V3.forward (v3.py:606-709): the reference's own feature
                   passes, then the decision trunk on the library's fp32 kernels (V3Trunk) from the model's own trunk
                   parameters.
  layouts          unchanged: Int8Linear's qweight/scale, PackedCache.tensors[(layer, "keys"|"values", None)].

    from opendecider.decider import Decider, prepare_inference_
    from opendecider_b200.integrate import prepare_b200_
    prepare_inference_(model)       # the reference's serving set-up
    prepare_b200_(model)            # then the B200 kernels; undo_b200_(model) restores the reference's paths

Everything else in the reference's forward (embedding, RMSNorm, RoPE, the state pass's SDPA, the readout) runs as
the reference runs it. A CPU model is refused (no CPU fallback).
"""
from __future__ import annotations

import contextlib
import types

import torch
import torch.nn.functional as F

from . import _lib
from .quant import W8A8


class PaddedW8A8(torch.nn.Module):
    """W8A8 for a linear whose shape the GEMM does not tile directly (K % 128 or N % 32 not zero, e.g. the tiny
    backbone's SwiGLU width 688): the int8 weight is padded once with zero columns / rows (scale 1), the activation
    with zero columns per call (zeros change neither its absmax nor any product), and the extra outputs dropped.
    Exact; holds its own padded copy of the weight."""

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, bias=None, inv_s=None):
        super().__init__()
        N, K = qweight.shape
        Np, Kp = -(-N // 32) * 32, -(-K // 128) * 128
        q = torch.zeros(Np, Kp, dtype=torch.int8, device=qweight.device)
        q[:N, :K] = qweight
        s = torch.ones(Np, dtype=torch.bfloat16, device=qweight.device)
        s[:N] = scale.reshape(-1).to(torch.bfloat16)
        iv = None
        if inv_s is not None:
            iv = torch.ones(Kp, dtype=torch.bfloat16, device=qweight.device)
            iv[:K] = inv_s.reshape(-1)
        self.inner = W8A8(q, s, None, iv)
        self.N, self.K, self.Kp, self.bias = N, K, Kp, bias
        self.in_features, self.out_features = K, N
        self._qweight, self._scale = qweight, scale

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.Kp != self.K:
            x = F.pad(x, (0, self.Kp - self.K))
        y = self.inner(x)[..., : self.N]
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y

    def dense_weight(self) -> torch.Tensor:
        return (self._qweight.to(self._scale.dtype) * self._scale.reshape(-1, 1)).t()


def _kernel_for(q: torch.Tensor, scale: torch.Tensor, bias):
    N, K = q.shape
    if N % 32 == 0 and K % 128 == 0:
        return W8A8(q, scale, bias)
    return PaddedW8A8(q, scale, bias)


def install_gemm_kernels_(module: torch.nn.Module) -> int:
    """Every int8 linear under `module` (anything with an int8 `qweight` and a `scale`, not training-materialised)
    gets a W8A8 `_fused` kernel on its own weight bytes. Returns how many."""
    n = 0
    for _, m in module.named_modules():
        q = getattr(m, "qweight", None)
        if isinstance(q, torch.Tensor) and q.dtype == torch.int8 and q.numel() and hasattr(m, "scale") \
                and m.__dict__.get("_dq") is None:
            if not q.is_cuda:
                raise _lib.ODError("prepare_b200_: the model must be on a CUDA device (there is no CPU path)")
            m.__dict__["_b200_prev_fused"] = m.__dict__.get("_fused")
            m.__dict__["_fused"] = _kernel_for(q, m.scale, getattr(m, "bias", None))
            n += 1
    return n


# ------------------------------------------------------------------------------------------------ attention seam
def _attn_modules(bb):
    return [(i, l.self_attn) for i, l in enumerate(bb.lm.layers)
            if bb.layer_types[i] == "full_attention" and hasattr(l, "self_attn")]


def _prefix(t):
    """A PackedCache tensor (the reference's Int8Tensor (S, Hkv, T, D) + scale (S, Hkv, T, 1), or a bf16 tensor when
    the K/V cache is not quantised) -> (K, scale (S, Hkv, T) or None)."""
    if hasattr(t, "q") and hasattr(t, "scale"):
        return t.q, t.scale.reshape(t.q.shape[:-1])
    return t, None


def _forward(mod, ctx, hidden_states, position_embeddings, attention_mask=None, past_key_values=None, **kw):
    """Qwen3_5Attention's math as the reference's prefix_attn._forward (prefix_attn.py:79-131: gated q, q/k RMSNorm,
    RoPE, output gate; projections through their modules, so their hooks run), with the attention in od_prefix_attn
    over the int8 state prefix (+ the question level) and the row's own keys."""
    from transformers.models.qwen3_5.modeling_qwen3_5 import apply_rotary_pos_emb
    R, t, _ = hidden_states.shape
    D = mod.head_dim
    q, gate = torch.chunk(mod.q_proj(hidden_states).view(R, t, -1, D * 2), 2, dim=-1)
    gate = gate.reshape(R, t, -1)
    q = mod.q_norm(q)                                                          # (R, t, Hq, D)
    k = mod.k_norm(mod.k_proj(hidden_states).view(R, t, -1, D))                 # (R, t, Hkv, D)
    v = mod.v_proj(hidden_states).view(R, t, -1, D)
    cos, sin = position_embeddings
    q, k = apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=2)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    li = mod.layer_idx
    if ctx["capture"] is not None:        # the question pass's own K/V, in the reference's (R, Hkv, t, D) shape
        ctx["capture"][li] = (k.transpose(1, 2), v.transpose(1, 2))
    Kp, ksc = _prefix(ctx["pc"].tensors[(li, "keys", None)])
    Vp, vsc = _prefix(ctx["pc"].tensors[(li, "values", None)])
    kw = dict(Kp=Kp, Vp=Vp, ksc=ksc, vsc=vsc, row_state=ctx["row_state"], pmask=ctx["pmask"], p_lo=ctx["p_lo"])
    if ctx["q_kv"] is not None:                                                # the question level
        Kq, Vq = ctx["q_kv"][li]
        kw.update(Kq=Kq.transpose(1, 2).contiguous(), Vq=Vq.transpose(1, 2).contiguous(), row_q=ctx["row_q"],
                  q_len=ctx["q_len"])
    o = _lib.prefix_attn(q, k, v, mod.scaling, **kw)
    o = o.reshape(R, t, -1) * torch.sigmoid(gate)
    return mod.o_proj(o), None


@contextlib.contextmanager
def b200_shared_prefix_attention(bb, pc, rows: torch.Tensor, pmask: torch.Tensor, static: bool = False,
                                 capture: dict | None = None, q_kv: dict | None = None,
                                 q_state: torch.Tensor | None = None):
    """The reference's shared_prefix_attention (prefix_attn.py:135-175), same arguments and meaning: while active,
    full-attention layers attend pc's per-state K/V for rows `rows` (row i reads state rows[i]); pmask (S, T) marks
    real prefix tokens; capture receives each layer's own (k, v); q_kv / q_state add the question level (rows then
    index questions, pmask (questions, T + Lq) covers both levels). static needs no special case: pads are masked
    in the kernel either way."""
    dev = rows.device
    mods = _attn_modules(bb)
    K0 = _prefix(pc.tensors[(mods[0][0], "keys", None)])[0]          # (S, Hkv, T, D)
    S, T = K0.shape[0], K0.shape[2]
    pm = pmask.bool()
    if q_kv is not None:
        qs = q_state.to(dev).long()
        smask = torch.zeros(S, T, dtype=torch.bool, device=dev)
        smask[qs] = pm[:, :T]                         # questions of one state carry that state's mask
        row_q = rows.to(dev).to(torch.int32)
        row_state = qs[rows.long()].to(torch.int32)
        q_len = pm[:, T:].sum(1).to(torch.int32)      # the question level is right-padded
    else:
        smask, row_q, q_len = pm, None, None
        row_state = rows.to(dev).to(torch.int32)
    p_lo = smask.to(torch.int8).argmax(1).to(torch.int32)   # first real key of each state (leading pads)
    ctx = {"pc": pc, "row_state": row_state, "pmask": smask.to(torch.uint8).contiguous(), "p_lo": p_lo,
           "capture": capture, "q_kv": q_kv, "row_q": row_q, "q_len": q_len}
    for _, m in mods:
        m.forward = types.MethodType(lambda self, *a, **k: _forward(self, ctx, *a, **k), m)
    try:
        yield
    finally:
        for _, m in mods:
            del m.forward


_TRUNK_PREFIXES = ("layer_mix", "in_norm.", "proj_", "layers.", "cls", "final_norm.", "score.", "rel.", "lp_proj.",
                   "lm_skip")


def _trunk_config(model):
    """The TrunkConfig of a reference V3 model whose trunk V3Trunk runs as the reference does - branched answer rows
    cross-attending the question only, the softmax layer mix, no context layers or context update, readout "last",
    no `none` sink, no slot embeddings - else None (that model keeps the reference's trunk)."""
    from .v3 import TrunkConfig
    cfg, bb = getattr(model, "cfg", None), getattr(model, "backbone", None)
    ok = (cfg is not None and bb is not None and getattr(cfg, "variant", None) == "v3"
          and getattr(model, "branched", False) and getattr(model, "state_free", False)
          and cfg.v3_layer_combine == "mix" and not cfg.v3_context_update and cfg.v3_context_layers == 0
          and cfg.v3_readout == "last" and not cfg.v3_none and cfg.slot_emb == "none")
    if not ok:
        return None
    return TrunkConfig(d_feat=model.d, n_feat_layers=len(bb.cfg.feature_layers), d_model=cfg.d_model,
                       n_heads=cfg.n_heads, decision_layers=cfg.decision_layers, lm_feature=bool(cfg.v3_lm_feature))


def b200_v3_forward(self, p, mem, questions=None, feats=None):
    """V3.forward (v3.py:606-709) of a reference model in the configuration _trunk_config accepts, with its trunk on
    the library's kernels: the reference's own frozen-LLM features (`_conditioned_feats_raw`: state pass, question
    cache, option rows, the LM feature), then V3Trunk on them - the layout V3.forward builds (option and question
    tokens, option ids, positions after the state), the layer mix, the decision layers, the CLS readout, `score` and
    `rel`. Calls with precomputed `feats` take the reference's own forward."""
    if feats is not None or questions is None:
        return type(self).forward(self, p, mem, questions, feats)
    from opendecider.models import DecisionOutput
    trunk = self.__dict__["_b200_trunk"]
    _, s_lens, q_flat, q_lens, o_flat, o_lens = self._conditioned_feats_raw(questions, mem)
    n_opt = torch.tensor([len(q.options) for q in questions])
    sidx = torch.tensor([q.state_idx for q in questions])
    plan = trunk.prepare(q_lens, o_lens, n_opt, s_lens[sidx])
    lp = self._lm_lp if trunk.cfg.lm_feature else None
    logits, rel = trunk.run(plan, q_flat, o_flat, lp, want_rel=True)
    return DecisionOutput(logits, p.opt_mask, rel, None)


def install_trunk_(model) -> int:
    """Give a reference V3 model the library's trunk (b200_v3_forward in place of its forward; the weights are the
    model's own trunk parameters, read once). Returns 1 if installed, 0 if the model's configuration is not one
    V3Trunk runs."""
    from .v3 import V3Trunk
    tc = _trunk_config(model)
    if tc is None or "_b200_trunk" in model.__dict__:
        return 0
    dev = model.backbone.device
    params = {k: v.detach() for k, v in model.state_dict().items() if k.startswith(_TRUNK_PREFIXES)}
    model.__dict__["_b200_trunk"] = V3Trunk(tc, params, dev)
    model.__dict__["forward"] = types.MethodType(b200_v3_forward, model)
    return 1


def prepare_b200_(model) -> dict:
    """Install the B200 kernels into a reference DecisionModel (its `.backbone` a reference Backbone on CUDA): the W8A8
    GEMM in every int8 linear's `_fused` slot, the int8-KV shared-prefix attention in place of the reference's
    shared_prefix_attention, and - for a V3 model in the serving configuration - the trunk (install_trunk_).
    Returns {"gemm": linears given a kernel, "attention": seams swapped, "trunk": trunks installed}."""
    import opendecider.v3 as ref_v3
    bb = model.backbone
    n = install_gemm_kernels_(bb.lm.layers)
    swapped = 0
    if getattr(ref_v3, "shared_prefix_attention", None) is not b200_shared_prefix_attention:
        model.__dict__["_b200_prev_attention"] = ref_v3.shared_prefix_attention
        ref_v3.shared_prefix_attention = b200_shared_prefix_attention
        swapped = 1
    return {"gemm": n, "attention": swapped, "trunk": install_trunk_(model)}


def undo_b200_(model) -> None:
    """Restore the reference's own kernels (the `_fused` slots as they were, its shared_prefix_attention)."""
    import opendecider.v3 as ref_v3
    for _, m in model.backbone.lm.layers.named_modules():
        if "_b200_prev_fused" in m.__dict__:
            prev = m.__dict__.pop("_b200_prev_fused")
            if prev is None:
                m.__dict__.pop("_fused", None)
            else:
                m.__dict__["_fused"] = prev
    prev = model.__dict__.pop("_b200_prev_attention", None)
    if prev is not None:
        ref_v3.shared_prefix_attention = prev
    if model.__dict__.pop("_b200_trunk", None) is not None:
        model.__dict__.pop("forward", None)
