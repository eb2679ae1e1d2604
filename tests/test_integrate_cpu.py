"""Host logic of the drop-in's attention seam (opendecider_b200.integrate.b200_shared_prefix_attention) on the CPU:
the reference's own decide_many (config 1, question cache on) with the reference's shared_prefix_attention replaced
by the drop-in's, whose od_prefix_attn call is answered here by a CPU restatement of that entry point's contract
(the int8 state prefix dequantised as materialize() does, pmask / p_lo, the question level up to q_len, the row's own
keys causally; the oracle's fp32 _split_attention). It checks how the drop-in maps the reference's arguments - rows,
pmask, capture, q_kv, q_state - onto the kernel's: the probabilities match the reference's golden within 1e-3.
The kernel itself is checked on the GPU (tests/test_integrate_gpu.py, tests/test_kernels_gpu.py).

The reference package is imported from baseline/_ref; without it the test is skipped."""
import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "baseline", "_ref")


def _attn_contract(q, k_own, v_own, sm_scale, *, Kp=None, Vp=None, ksc=None, vsc=None, row_state=None, p_lo=None,
                   pmask=None, Kq=None, Vq=None, row_q=None, q_len=None, **_):
    from oracle import ops
    R, t, Hq, D = q.shape
    out = torch.empty(R, t, Hq, D, dtype=torch.bfloat16)
    for r in range(R):
        s = int(row_state[r])
        K = ops.materialize_int8(Kp[s], ksc[s][..., None])           # (Hkv, T, D)
        V = ops.materialize_int8(Vp[s], vsc[s][..., None])
        pm = pmask[s].bool() & (torch.arange(K.shape[1]) >= int(p_lo[s]))
        if Kq is not None:
            j = int(row_q[r])
            K = torch.cat([K, Kq[j].transpose(0, 1)], 1)
            V = torch.cat([V, Vq[j].transpose(0, 1)], 1)
            pm = torch.cat([pm, torch.arange(Kq.shape[1]) < int(q_len[j])])
        o = ops.split_attention(q[r:r + 1].transpose(1, 2), k_own[r:r + 1].transpose(1, 2),
                                v_own[r:r + 1].transpose(1, 2), K, V, pm, sm_scale)
        out[r] = o[0].transpose(0, 1).to(torch.bfloat16)
    return out


def test_drop_in_attention_seam_maps_the_reference_arguments(monkeypatch):
    if not os.path.isdir(os.path.join(REF, "opendecider")):
        pytest.skip("the reference package is not installed in baseline/_ref")
    os.environ["OPENDECIDER_REF"] = REF
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from make_golden_e2e import FEATURE_LAYERS, TEMPS, TRUNK, build_reference, use_reference
    use_reference()
    from opendecider.decider import Decider, prepare_inference_
    from opendecider.models import ModelConfig, build_model
    import opendecider.v3 as ref_v3
    from opendecider_b200 import integrate
    from opendecider_b200 import synthetic as syn
    from opendecider_b200.backbone import DecoderConfig
    from opendecider_b200.v3 import TrunkConfig, trunk_state_dict

    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    reqs, tok = syn.decision_requests(1, seed=0)
    bb = build_reference(cfg, tok)
    mcfg = ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched", v3_row_format="answer",
                       v3_cross="question", v3_layer_combine="mix", **TRUNK)
    model = build_model(bb, mcfg).eval()
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    model.load_state_dict(trunk_state_dict(tc, seed=0), strict=False)
    monkeypatch.setenv("OPENDECIDER_QCACHE", "1")
    prepare_inference_(model)
    calls = []
    monkeypatch.setattr(integrate._lib, "prefix_attn",
                        lambda *a, **k: calls.append(k.get("Kq") is not None) or _attn_contract(*a, **k))
    monkeypatch.setattr(ref_v3, "shared_prefix_attention", integrate.b200_shared_prefix_attention)
    dec = Decider(model, temperature=1.419344425201416, temperature_by_type=TEMPS)
    dreqs = [{"state": r.state, "questions": {q.name: {"type": q.type, "prompt": q.prompt, "options": q.options}
                                              for q in r.questions}} for r in reqs]
    with torch.no_grad():
        ans = dec.decide_many(dreqs)
    assert calls and any(calls) and not all(calls)          # question pass (one level) and option rows (two)
    g = np.load(os.path.join(HERE, "golden", "e2e_config1.npz"))
    p = np.array([a["answers"]["q0"]["probs_list"] for a in ans])
    assert np.abs(p - g["qcache.probs"]).max() < 1e-3, np.abs(p - g["qcache.probs"]).max()
