"""Golden decisions of a SmoothQuant (a8w8sq) tiny model, produced by the REFERENCE's own Decider.decide_many on CPU
(the backbone and trunk of make_golden_e2e.py, question cache on, BASELINE config 1's requests):

  1. calibration as the reference's scripts/smoothquant_calibrate.py does it: the bf16 model (weight_quant none)
     decides calibration requests (decision_requests(1, seed=11)) while forward pre-hooks record max |x| per input
     channel of every linear under the layer list;
  2. scales: the reference's own smooth_scales(amax, W, alpha) (quant.py:353-356) per linear, alpha 0.65 (the value
     its RESULTS picked for the served 9B);
  3. the smoothed model (make_golden_e2e.build_reference(smooth=...): the reference's Int8Linear / SmoothedLinear
     classes with the A8W8 arithmetic at the _fused seam) decides config 1.

Writes tests/golden/smooth_config1.npz: per request the renormalised probabilities (`probs`), P(none) (`none`),
the trunk logits (`logits`) and every scale vector (`scale.<name>`, fp32, name relative to the layer list).

    OPENDECIDER_REF=<reference>/src python tests/golden/make_golden_smooth.py
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden_e2e import FEATURE_LAYERS, TEMPS, TRUNK, build_reference, use_reference  # noqa: E402

from opendecider_b200 import synthetic as syn  # noqa: E402
from opendecider_b200.backbone import DecoderConfig  # noqa: E402
from opendecider_b200.v3 import TrunkConfig, trunk_state_dict  # noqa: E402

ALPHA = 0.65
CALIB_SEED = 11


def decider(bb, cfg):
    from opendecider.decider import Decider, prepare_inference_
    from opendecider.models import ModelConfig, build_model
    mcfg = ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched", v3_row_format="answer",
                       v3_cross="question", v3_layer_combine="mix", **TRUNK)
    model = build_model(bb, mcfg).eval()
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    missing, unexpected = model.load_state_dict(trunk_state_dict(tc, seed=0), strict=False)
    assert not unexpected, unexpected
    os.environ["OPENDECIDER_QCACHE"] = "1"
    prepare_inference_(model)
    return Decider(model, temperature=1.419344425201416, temperature_by_type=TEMPS), model


def as_dicts(reqs):
    return [{"state": r.state, "questions": {q.name: {"type": q.type, "prompt": q.prompt, "options": q.options}
                                             for q in r.questions}} for r in reqs]


def calibrate(cfg):
    """max |x| per input channel of every linear under the layer list, over the calibration requests."""
    import torch.nn as nn
    from opendecider.quant import smooth_scales
    calib, tok = syn.decision_requests(1, seed=CALIB_SEED)
    bb = build_reference(cfg, tok, quantize=False)
    amax, hooks = {}, []
    for name, mod in bb.lm.layers.named_modules():
        if isinstance(mod, nn.Linear):
            def hook(m, args, name=name):
                x = args[0].detach().reshape(-1, args[0].shape[-1]).abs().amax(0).float()
                amax[name] = x if name not in amax else torch.maximum(amax[name], x)
            hooks.append(mod.register_forward_pre_hook(hook))
    dec, _ = decider(bb, cfg)
    with torch.no_grad():
        dec.decide_many(as_dicts(calib))
    for h in hooks:
        h.remove()
    W = {name: mod.weight.data for name, mod in bb.lm.layers.named_modules() if isinstance(mod, nn.Linear)}
    return {n: smooth_scales(amax[n], W[n], ALPHA).cpu() for n in amax}


def main():
    use_reference()
    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    scales = calibrate(cfg)
    reqs, tok = syn.decision_requests(1, seed=0)
    bb = build_reference(cfg, tok, smooth=scales)
    dec, model = decider(bb, cfg)
    from opendecider import v3 as ref_v3
    logits = []
    orig = ref_v3.V3.forward

    def rec(self, *a, **k):
        out = orig(self, *a, **k)
        logits.append(out.logits.detach().clone())
        return out

    ref_v3.V3.forward = rec
    try:
        with torch.no_grad():
            ans = dec.decide_many(as_dicts(reqs))
    finally:
        ref_v3.V3.forward = orig
    K = max(len(q.options) for r in reqs for q in r.questions)
    probs = np.zeros((len(reqs), K), dtype=np.float64)
    none = np.zeros(len(reqs), dtype=np.float64)
    for i, a in enumerate(ans):
        pl = a["answers"]["q0"]["probs_list"]
        probs[i, : len(pl)] = pl
        none[i] = a["answers"]["q0"]["none"]
    out = {"probs": probs, "none": none, "logits": logits[0].numpy()}
    out.update({f"scale.{n}": v.numpy().astype(np.float32) for n, v in scales.items()})
    np.savez_compressed(os.path.join(HERE, "smooth_config1.npz"), **out)
    print(probs.round(4), none.round(4), len(scales), "scale vectors")


if __name__ == "__main__":
    main()
