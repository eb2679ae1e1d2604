"""The CPU oracle of the whole decision forward (oracle/model.py, the timed CPU baseline) reproduces the reference's
own Decider.decide_many (tests/golden/e2e_config1.npz, tests/golden/edge_cases.npz) bit for bit on the machine that
made the fixtures: it routes every attention call as the reference does (the transformers SDPA call of the state pass,
shared_prefix_attention's one-call multi-state path or its per-state _split_attention) and makes the same CPU calls.
The bound 1e-6 only leaves room for another CPU's vector width in torch's attention kernel.

The last test measures how sensitive the edge batch's yes/no question is to the last bit of attention: the same
oracle with one change inside attention - torch.exp in place of the CPU kernel's own exponential, a division in place
of its reciprocal multiply (one-ulp changes of the bf16 attention output on about 9 % of its elements) - moves that
question's probabilities by more than 1e-3. An attention that is not bit-identical to torch's CPU kernel, such as a
tensor-core kernel, cannot be held to 1e-3 there."""
import numpy as np

from oracle.model import OracleDecision
from oracle.trunk import OracleTrunk
from opendecider_b200 import synthetic as syn
from opendecider_b200.backbone import DecoderConfig, synthetic_weights
from opendecider_b200.v3 import TrunkConfig, trunk_state_dict

FEATURE_LAYERS = (1, 3, "final")
TRUNK = dict(d_model=64, n_heads=4, decision_layers=2)
TEMPS = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}


def test_oracle_decide_matches_reference():
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
    reqs, tok = syn.decision_requests(1, seed=0)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), trunk, tok, TEMPS, 1.419344425201416,
                        qcache_min_rows=32)
    probs, ren, pn, logits = od.decide(reqs)
    g = np.load("tests/golden/e2e_config1.npz")
    K = g["qcache.probs"].shape[1]
    assert np.abs(ren[:, :K] - g["qcache.probs"]).max() < 1e-6
    assert np.abs(pn - g["qcache.none"]).max() < 1e-6
    assert np.abs(logits.numpy() - g["qcache.logits"]).max() < 1e-5


def test_oracle_lm_feature_matches_reference():
    """The V3 trunk's LM log-prob feature (v3_lm_feature): the oracle's token_logprob over the tied int8 head and the
    trunk's lp_proj / gated skip reproduce the reference's decide_many (the feature moves the probabilities by up to
    1.2e-2 on this case, so the check discriminates)."""
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), lm_feature=True, **TRUNK)
    trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
    reqs, tok = syn.decision_requests(1, seed=0)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), trunk, tok, TEMPS, 1.419344425201416,
                        qcache_min_rows=32)
    probs, ren, pn, logits = od.decide(reqs)
    g = np.load("tests/golden/e2e_config1.npz")
    K = g["lmq.probs"].shape[1]
    assert np.abs(ren[:, :K] - g["lmq.probs"]).max() < 1e-6
    assert np.abs(pn - g["lmq.none"]).max() < 1e-6
    assert np.abs(logits.numpy() - g["lmq.logits"]).max() < 1e-5


def _edge_oracle(sdpa=None):
    import sys
    sys.path.insert(0, "tests/golden")
    from make_golden_edge import NAMES, edge_requests
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
    tok = syn.SyntheticTokenizer(cfg.vocab)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), trunk, tok, TEMPS, 1.419344425201416,
                        qcache_min_rows=32, sdpa=sdpa)
    _, ren, pn, _ = od.decide(edge_requests())
    g = np.load("tests/golden/edge_cases.npz")
    return {name: float(np.abs(ren[i, : g[f"{name}.probs"].size] - g[f"{name}.probs"]).max())
            for i, name in enumerate(NAMES)}


def test_oracle_edge_cases_match_reference():
    """The edge batch (tests/golden/edge_cases.npz: ragged left-padded states, 255 options, yes/no, a right-padded
    question pass reading three states through one masked call): the oracle equals the reference."""
    for name, d in _edge_oracle().items():
        assert d < 1e-6, (name, d)


def test_edge_yes_no_is_sensitive_to_the_last_bit_of_attention():
    """The oracle with one change inside its attention calls (oracle.model.sdpa_exp_variant: torch.exp for the CPU
    kernel's exponential, a division for its reciprocal multiply) moves the yes/no question of the edge batch by
    more than 1e-3 from the reference - so 1e-3 on that question demands an attention bit-identical to torch's CPU
    kernel - while the 255-option question stays within 1e-4."""
    from oracle.model import sdpa_exp_variant
    d = _edge_oracle(sdpa_exp_variant)
    assert d["yn"] > 1e-3, d
    assert d["big"] < 1e-4, d


def smooth_scales_from_golden(g) -> dict:
    """The SmoothQuant scales the golden was made with ({'{i}.self_attn.q_proj': s, ...}, fp32)."""
    import torch
    return {k[len("scale."):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("scale.")}


def test_oracle_smoothquant_matches_reference():
    """A8 row A3: a SmoothQuant model (the reference's smooth_a8w8_ folding + SmoothedLinear, calibrated scales per
    linear, alpha 0.65: tests/golden/smooth_config1.npz) decided by the oracle equals the reference's decide_many."""
    g = np.load("tests/golden/smooth_config1.npz")
    scales = smooth_scales_from_golden(g)
    assert len(scales) == 28                               # 7 linears x 4 layers, each its own vector
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
    reqs, tok = syn.decision_requests(1, seed=0)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), trunk, tok, TEMPS, 1.419344425201416,
                        qcache_min_rows=32, smooth=scales)
    _, ren, pn, logits = od.decide(reqs)
    K = g["probs"].shape[1]
    assert np.abs(ren[:, :K] - g["probs"]).max() < 1e-6
    assert np.abs(pn - g["none"]).max() < 1e-6
    assert np.abs(logits.numpy() - g["logits"]).max() < 1e-5
    # the smoothing moves the trunk logits by 1e-2 (this random-init model has no activation outliers to move)
    base = np.load("tests/golden/e2e_config1.npz")["qcache.logits"]
    assert np.abs(g["logits"] - base).max() > 5e-3
