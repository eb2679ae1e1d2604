"""Golden answers of edge-case requests, produced by the REFERENCE's own Decider.decide_many on CPU (the tiny
backbone and trunk of make_golden_e2e.py, question cache on): ragged states (7, 300 and 45 tokens: a left-padded
state pass), a question at the 255-option cap (no `none` option), a two-option choice, a yes/no question (the
reference supplies its options) and a three-option choice. Writes tests/golden/edge_cases.npz: per question the
renormalised probabilities (`{name}.probs`) and P(none) (`{name}.none`, NaN when the question has none)."""
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
from opendecider_b200.batching import Question  # noqa: E402
from opendecider_b200.v3 import TrunkConfig, trunk_state_dict  # noqa: E402

NAMES = ["big", "two", "yn", "small"]


def edge_requests():
    """The edge batch (seeded; shared with the tests)."""
    g = syn.gen(77)
    ids = lambda n: syn.words(torch.randint(16, 1024, (n,), generator=g).tolist())
    big = [ids(2) for _ in range(255)]
    return [syn.Request(ids(4), [Question(ids(6), big, "choice", name="big")]),
            syn.Request(ids(297), [Question(ids(5), [ids(3), ids(1)], "choice", name="two"),
                                   Question.noul(ids(4), name="yn")]),
            syn.Request(ids(42), [Question(ids(3), [ids(2), ids(5), ids(1)], "choice", name="small")])]


def main():
    use_reference()
    from opendecider.decider import Decider, prepare_inference_
    from opendecider.models import ModelConfig, build_model
    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    tok = syn.SyntheticTokenizer(cfg.vocab)
    reqs = edge_requests()
    bb = build_reference(cfg, tok)
    mcfg = ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched", v3_row_format="answer",
                       v3_cross="question", v3_layer_combine="mix", **TRUNK)
    model = build_model(bb, mcfg).eval()
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    missing, unexpected = model.load_state_dict(trunk_state_dict(tc, seed=0), strict=False)
    assert not unexpected, unexpected
    os.environ["OPENDECIDER_QCACHE"] = "1"
    prepare_inference_(model)
    dec = Decider(model, temperature=1.419344425201416, temperature_by_type=TEMPS)
    dreqs = [{"state": r.state, "questions": {
        q.name: ({"type": q.type, "prompt": q.prompt} if q.type == "noul" else
                 {"type": q.type, "prompt": q.prompt, "options": q.options}) for q in r.questions}} for r in reqs]
    ans = dec.decide_many(dreqs)
    out = {}
    for i, r in enumerate(reqs):
        for q in r.questions:
            a = ans[i]["answers"][q.name]
            out[f"{q.name}.probs"] = np.array(a["probs_list"], dtype=np.float64)
            out[f"{q.name}.none"] = np.float64(a.get("none", np.nan))
    np.savez_compressed(os.path.join(HERE, "edge_cases.npz"), **out)
    print({k: v.round(4)[:4] if v.ndim else v for k, v in out.items()})


if __name__ == "__main__":
    main()
