"""The drop-in (opendecider_b200.integrate.prepare_b200_) on the REFERENCE's own model: the reference's tiny Decider
(the set-up of tests/golden/make_golden_e2e.py: its Qwen3.5 backbone with Int8Linear / Int8Embedding, its V3 trunk,
prepare_inference_ with the question cache) built on CUDA, then the B200 kernels installed at the reference's seams -
the W8A8 GEMM in every Int8Linear's `_fused` slot, the int8-KV shared-prefix attention in place of
shared_prefix_attention, the decision trunk in place of V3.forward's (b200_v3_forward). Its decide_many on BASELINE config 1 must match the golden of the reference's own CPU run
(tests/golden/e2e_config1.npz) within 1e-3, with forward hooks on the int8 linears (how the reference's VeRA adapters
attach, vera.py:54) still firing, and the library's kernels doing the work.

The reference package is imported from baseline/_ref (a pip install of the reference made next to this repository);
without it the test is skipped."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "baseline", "_ref")

pytestmark = pytest.mark.gpu


def test_prepare_b200_on_the_reference_decider(cuda):
    if not os.path.isdir(os.path.join(REF, "opendecider")):
        pytest.skip("the reference package is not installed in baseline/_ref")
    os.environ["OPENDECIDER_REF"] = REF
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from make_golden_e2e import FEATURE_LAYERS, TEMPS, TRUNK, build_reference, use_reference
    use_reference()
    from opendecider.decider import Decider, prepare_inference_
    from opendecider.models import ModelConfig, build_model
    import opendecider.v3 as ref_v3
    from opendecider_b200 import _lib
    from opendecider_b200 import synthetic as syn
    from opendecider_b200.backbone import DecoderConfig
    from opendecider_b200.integrate import b200_shared_prefix_attention, prepare_b200_, undo_b200_
    from opendecider_b200.v3 import TrunkConfig, trunk_state_dict

    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    reqs, tok = syn.decision_requests(1, seed=0)
    bb = build_reference(cfg, tok, device="cuda")
    mcfg = ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched", v3_row_format="answer",
                       v3_cross="question", v3_layer_combine="mix", **TRUNK)
    model = build_model(bb, mcfg).eval()
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    model.load_state_dict(trunk_state_dict(tc, seed=0), strict=False)
    model.to(cuda)
    os.environ["OPENDECIDER_QCACHE"] = "1"
    prepare_inference_(model)
    got = prepare_b200_(model)
    try:
        assert got == {"gemm": 7 * cfg.layers, "attention": 1, "trunk": 1}
        assert ref_v3.shared_prefix_attention is b200_shared_prefix_attention
        assert "_b200_trunk" in model.__dict__ and "forward" in model.__dict__
        calls = [0]
        hook = bb.lm.layers[1].self_attn.q_proj.register_forward_hook(
            lambda m, a, out: calls.__setitem__(0, calls[0] + 1))
        l0 = _lib.LAUNCHES[0]
        _lib.KERNEL_PROBE = {}
        dec = Decider(model, temperature=1.419344425201416, temperature_by_type=TEMPS)
        dreqs = [{"state": r.state, "questions": {q.name: {"type": q.type, "prompt": q.prompt, "options": q.options}
                                                  for q in r.questions}} for r in reqs]
        with torch.no_grad():
            ans = dec.decide_many(dreqs)
        torch.cuda.synchronize()
        hook.remove()
        assert calls[0] >= 3                           # state pass, question pass, option rows
        assert _lib.LAUNCHES[0] - l0 > 50              # the GEMMs and attention ran in libod_b200
        ran = set(_lib.KERNEL_PROBE)
        assert {"gemm_f32", "trunk_attn", "scalenorm_split", "xatglu_split"} <= ran, ran   # the trunk too
        assert _lib.device_error(cuda) == 0
    finally:
        _lib.KERNEL_PROBE = None
        undo_b200_(model)
    assert ref_v3.shared_prefix_attention is not b200_shared_prefix_attention
    assert "_b200_trunk" not in model.__dict__ and "forward" not in model.__dict__
    g = np.load(os.path.join(HERE, "golden", "e2e_config1.npz"))
    p = np.array([a["answers"]["q0"]["probs_list"] for a in ans])
    none = np.array([a["answers"]["q0"]["none"] for a in ans])
    assert np.abs(p - g["qcache.probs"]).max() < 1e-3, np.abs(p - g["qcache.probs"]).max()
    assert np.abs(none - g["qcache.none"]).max() < 1e-3
