"""Golden decision probabilities of BASELINE config 1, produced by the REFERENCE implementation's own
Decider.decide_many (src/opendecider/decider.py:438-484) on CPU in bf16.

Reference set-up (only the shims the reference needs to run here, none of which changes its arithmetic):
  - Qwen3_5ForCausalLM with every layer `full_attention` (hidden 256, 4 layers, 4 q / 2 kv heads, head_dim 64,
    SwiGLU 688, vocab 1024, rope_theta 1e6 with partial_rotary_factor pinned to 1.0), bf16, weights loaded from
    opendecider_b200.backbone.synthetic_weights(seed 0);
  - quantize_int8_ on the decoder layers and Int8Embedding on the table (the reference's own quantisers);
  - the A8W8 arithmetic at the reference's own kernel seam Int8Linear._fused (quant.py:150-152): per-token int8
    activations by the in-tree formula (Int8Tensor.quantize, quant.py:37-41, fp32 scale), exact int32 products,
    bf16((acc * s_x) * s_w). GemLite's A8W8 (the reference's GPU kernel, quant.py:302-314) is not vendored and not
    installed; this restates its arithmetic, so the W8A8 epilogue itself is unpinned by a reference run;
  - use_reference_kernels(True) and a no-op Qwen3_5TextModel._update_linear_attn_mask (transformers 5.5 raises on
    an all-attention cache otherwise);
  - the word-level SyntheticTokenizer (the Qwen tokenizer is not available offline);
  - a V3 model (branched answer rows, v3_cross="question", slot_emb none, d_model 64, 4 heads, 2 layers,
    feature layers [1, 3, final]) with trunk weights from opendecider_b200.v3.trunk_state_dict(seed 0), then
    prepare_inference_ (question cache on: 36 option rows >= the 32-row threshold).
Writes tests/golden/e2e_config1.npz: per question the renormalised probabilities and P(none), the trunk logits, for
the question-cache path and (OPENDECIDER_QCACHE=0) the one-row-per-option path.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from opendecider_b200 import synthetic as syn  # noqa: E402
from opendecider_b200.backbone import DecoderConfig, synthetic_weights  # noqa: E402
from opendecider_b200.v3 import TrunkConfig, trunk_state_dict  # noqa: E402

FEATURE_LAYERS = [1, 3, "final"]
TRUNK = dict(d_model=64, n_heads=4, decision_layers=2)
TEMPS = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}


class A8W8:
    """W8A8 arithmetic installed in Int8Linear._fused: per-token int8 x, exact int32 x int8 weight, bf16 epilogue."""

    def __init__(self, m):
        self.q, self.s = m.qweight, m.scale

    def __call__(self, x):
        shp = x.shape
        xf = x.reshape(-1, shp[-1]).float()
        s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 127.0
        q = torch.round(xf / s).clamp_(-127, 127).to(torch.int32)
        acc = q @ self.q.to(torch.int32).t()
        y = ((acc.float() * s) * self.s.float().view(1, -1)).to(x.dtype)
        return y.view(*shp[:-1], -1)

    def dense_weight(self):
        return (self.q.float() * self.s.float()).to(torch.bfloat16).t()


def use_reference() -> None:
    """Put the reference's src/ directory (OPENDECIDER_REF, required) on sys.path; the generators import it."""
    ref = os.environ.get("OPENDECIDER_REF")
    if not ref:
        sys.exit("set OPENDECIDER_REF to the reference checkout's src/ directory")
    if ref not in sys.path:
        sys.path.insert(0, ref)


def build_reference(cfg: DecoderConfig, tok, quantize: bool = True, smooth: dict | None = None, device: str = "cpu"):
    """The reference's tiny backbone. quantize=False: the bf16 model (weight_quant none, the SmoothQuant calibration
    model). smooth {'{i}.self_attn.q_proj': s, ...}: the reference's a8w8sq load (smooth_a8w8_, quant.py:333-350)
    restated around its own classes: W *= s per input channel (fp32 product, bf16 weight), the weight quantised by
    the reference's Int8Linear with the A8W8 arithmetic at its _fused seam (GemLite's A8W8 is not installed), and
    the reference's SmoothedLinear(inner, s) in the linear's place (x * inv_s before the product). device: where the
    model is placed after it is built and quantised (the goldens are made on the CPU; the drop-in test runs it on
    CUDA)."""
    use_reference()
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5TextModel
    from opendecider.backbone import Backbone, BackboneConfig, use_reference_kernels
    from opendecider.quant import Int8Embedding, Int8Linear, quantize_int8_
    use_reference_kernels(True)
    Qwen3_5TextModel._update_linear_attn_mask = lambda self, am, pkv: None
    c = Qwen3_5TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=cfg.layers,
        num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        layer_types=["full_attention"] * cfg.layers, rms_norm_eps=cfg.eps, tie_word_embeddings=True,
        pad_token_id=tok.pad_token_id,
        rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta, "partial_rotary_factor": 1.0})
    m = Qwen3_5ForCausalLM(c)
    inv_freq = m.model.rotary_emb.inv_freq.clone()
    m = m.to(torch.bfloat16).eval()
    lm = m.model
    # from_pretrained(dtype=bfloat16) - the reference's load path (backbone.py:118) - keeps the rotary inv_freq
    # buffer in fp32; a whole-module .to(bfloat16) would round it, so the fp32 buffer is put back.
    lm.rotary_emb.inv_freq = inv_freq
    missing, unexpected = lm.load_state_dict(synthetic_weights(cfg, seed=0), strict=False)
    assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
    if quantize:
        smooth = smooth or {}
        for name, mod in lm.layers.named_modules():
            if isinstance(mod, torch.nn.Linear) and name in smooth:
                s = smooth[name].to(torch.float32)
                mod.weight.data = (mod.weight.data.float() * s[None, :]).to(mod.weight.dtype)
        quantize_int8_(lm.layers)
        lm.embed_tokens = Int8Embedding(lm.embed_tokens)
        for mod in lm.layers.modules():
            if isinstance(mod, Int8Linear):
                mod.__dict__["_fused"] = A8W8(mod)
        if smooth:
            from opendecider.quant import SmoothedLinear
            for name, s in smooth.items():
                parent_name, attr = name.rsplit(".", 1)
                parent = lm.layers.get_submodule(parent_name)
                setattr(parent, attr, SmoothedLinear(getattr(parent, attr), s.to(torch.float32)))
    lm = lm.to(device)
    bcfg = BackboneConfig(path="synthetic", dtype="bfloat16", weight_quant="int8" if quantize else "none",
                          kv_quant="int8", feature_layers=list(FEATURE_LAYERS), device=device)
    return Backbone(lm, tok, bcfg)


def run(qcache: bool, lm: bool = False):
    use_reference()
    from opendecider.models import ModelConfig, build_model
    from opendecider.decider import Decider, prepare_inference_
    from opendecider import v3 as ref_v3
    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    reqs, tok = syn.decision_requests(1, seed=0)
    bb = build_reference(cfg, tok)
    mcfg = ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched", v3_row_format="answer",
                       v3_cross="question", v3_layer_combine="mix", v3_lm_feature=lm, **TRUNK)
    model = build_model(bb, mcfg).eval()
    sd = trunk_state_dict(TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), lm_feature=lm, **TRUNK),
                          seed=0)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    os.environ["OPENDECIDER_QCACHE"] = "1" if qcache else "0"
    prepare_inference_(model)
    logits = []
    orig = ref_v3.V3.forward

    def rec(self, *a, **k):
        out = orig(self, *a, **k)
        logits.append(out.logits.detach().clone())
        return out

    ref_v3.V3.forward = rec
    try:
        dec = Decider(model, temperature=1.419344425201416, temperature_by_type=TEMPS)
        dreqs = [{"state": r.state, "questions": {q.name: {"type": q.type, "prompt": q.prompt, "options": q.options}
                                                  for q in r.questions}} for r in reqs]
        ans = dec.decide_many(dreqs)
    finally:
        ref_v3.V3.forward = orig
    K = max(len(q.options) for r in reqs for q in r.questions)
    probs = np.zeros((len(reqs), K), dtype=np.float64)
    none = np.zeros(len(reqs), dtype=np.float64)
    for i, a in enumerate(ans):
        a = a["answers"]
        pl = a["q0"]["probs_list"]
        probs[i, : len(pl)] = pl
        none[i] = a["q0"]["none"]
    return probs, none, logits[0].numpy()


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}
    for qc, lm in ((True, False), (False, False), (True, True), (False, True)):
        p, n, lg = run(qc, lm)
        tag = ("lmq" if qc else "lmr") if lm else ("qcache" if qc else "rows")
        out[f"{tag}.probs"], out[f"{tag}.none"], out[f"{tag}.logits"] = p, n, lg
        print(tag, p.round(4), n.round(4))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "e2e_config1.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
