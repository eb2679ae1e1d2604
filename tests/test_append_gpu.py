"""Config 5 on the B200 path: cached states extended by appended tokens (PrefixCache.encode's continuation,
state_cache.py:116-158), then decided. Checked against the reference's own PrefixCache K/V
(tests/golden/append_config5.npz) and against the CPU oracle's decisions.

Bars: layer 0's appended K/V byte for byte (nothing float-ordered upstream of it); deeper layers within the
dequantised tolerance of the oracle's own pin (the attention summation order differs between implementations, and
int8 activation quantisation turns a one-ulp change into a step); probabilities within 1e-3 of the oracle; the three
ways of reading the prefix (kept bf16 copy, per-layer copy made for the pass, int8 dequantised inside attention)
bit-identical."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from make_golden_append import APPEND, N_REQ, OPTIONS, STATE  # noqa: E402

from opendecider_b200 import synthetic as syn  # noqa: E402
from opendecider_b200.backbone import Backbone, DecoderConfig, synthetic_weights  # noqa: E402
from opendecider_b200.decider import Decider  # noqa: E402
from opendecider_b200.v3 import TrunkConfig, V3Model, V3Trunk, trunk_state_dict  # noqa: E402

pytestmark = pytest.mark.gpu

FEATURE_LAYERS = (1, 3, "final")
TRUNK = dict(d_model=64, n_heads=4, decision_layers=2)
TEMPS = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}
TEMPERATURE = 1.419344425201416
CHAIN_REL_TOL = 0.06


def _requests(cfg):
    return syn.decision_requests(5, seed=3, n_requests=N_REQ, vocab=cfg.vocab, state_tokens=STATE,
                                 n_options=OPTIONS, append_tokens=APPEND)


def make(cuda):
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    reqs, tok = _requests(cfg)
    bb = Backbone.random(cfg, seed=0, device=cuda, gen_device="cpu")
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    trunk = V3Trunk(tc, trunk_state_dict(tc, seed=0), cuda)
    model = V3Model(bb, trunk, tok, question_cache=True, qcache_min_rows=32)
    return cfg, reqs, tok, Decider(model, temperature=TEMPERATURE, temperature_by_type=TEMPS)


def _deq(q, s):
    return q.astype(np.float32) * s.astype(np.float32)[..., None]


def _append(dec, reqs, tok, cuda):
    cache = dec.encode_states([r.state for r in reqs], cap=STATE + APPEND)
    ids = torch.tensor(tok([r.append for r in reqs], add_special_tokens=False)["input_ids"], device=cuda)
    dec.model.backbone.run_append(ids, cache)
    return cache


def test_append_kv_matches_reference_prefixcache(cuda):
    cfg, reqs, tok, dec = make(cuda)
    g = np.load(os.path.join(HERE, "golden", "append_config5.npz"))
    cache = _append(dec, reqs, tok, cuda)
    assert cache.T == STATE + APPEND and cache.lens == [STATE + APPEND] * N_REQ
    for r in range(N_REQ):
        for li in range(cfg.layers):
            for a, t in (("k", cache.k[li]), ("v", cache.v[li])):
                q8 = t.q[r, :, STATE:STATE + APPEND].cpu().numpy()
                sb = t.scale[r, :, STATE:STATE + APPEND].cpu().contiguous().view(torch.int16).numpy()
                gq, gs = g[f"snap.{r}.{li}.{a}.q"], g[f"snap.{r}.{li}.{a}.s"]
                if li == 0:
                    assert np.array_equal(q8, gq) and np.array_equal(sb, gs), (r, a)
                else:
                    f = lambda b: torch.from_numpy(b).view(torch.bfloat16).float().numpy()
                    ref = _deq(gq, f(gs))
                    rel = float(np.abs(_deq(q8, f(sb)) - ref).max() / np.abs(ref).max())
                    assert rel <= CHAIN_REL_TOL, (r, li, a, rel)


def test_append_matches_oracle_append(cuda):
    """The appended K/V of every layer against the oracle's continuation on the same inputs."""
    from oracle.model import OracleDecision
    cfg, reqs, tok, dec = make(cuda)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), None, tok, {}, 1.0)
    _, snaps, _ = od.append_pass(od.state_pass([r.state for r in reqs]), [r.append for r in reqs])
    cache = _append(dec, reqs, tok, cuda)
    for li in range(cfg.layers):
        for ai, t in enumerate((cache.k[li], cache.v[li])):
            q8 = t.q[:, :, STATE:STATE + APPEND].cpu().numpy()
            s = t.scale[:, :, STATE:STATE + APPEND].cpu().float().numpy()
            oq, os_ = snaps[li][ai]
            if li == 0:
                assert np.array_equal(q8, oq.numpy())
                assert np.array_equal(s, os_.float().numpy())
            else:
                ref = _deq(oq.numpy(), os_.float().numpy())
                rel = float(np.abs(_deq(q8, s) - ref).max() / np.abs(ref).max())
                assert rel <= CHAIN_REL_TOL, (li, ai, rel)


def _decide_cached(dec, reqs, cache):
    plan = dec.plan(reqs, cache=cache, appends=[r.append for r in reqs])
    probs, cache = dec.execute(plan, cache)
    return dec.answers(plan, probs)


def _flat(ans):
    p = np.array([a["choice"]["probs_list"] for a in ans])
    return p, np.array([a["choice"]["none"] for a in ans])


def test_append_decisions_match_oracle(cuda):
    from oracle.model import OracleDecision
    from oracle.trunk import OracleTrunk
    cfg, reqs, tok, dec = make(cuda)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), OracleTrunk(tc, trunk_state_dict(tc, seed=0)), tok,
                        TEMPS, TEMPERATURE, qcache_min_rows=32)
    nxt, _, _ = od.append_pass(od.state_pass([r.state for r in reqs]), [r.append for r in reqs])
    _, ren, pn, _ = od.decide(reqs, prebuilt=nxt)
    cache = dec.encode_states([r.state for r in reqs], cap=STATE + APPEND)
    p, none = _flat(_decide_cached(dec, reqs, cache))
    assert np.abs(p - ren[:, : p.shape[1]]).max() < 1e-3, np.abs(p - ren[:, : p.shape[1]]).max()
    assert np.abs(none - pn).max() < 1e-3


def test_append_replay_is_idempotent(cuda):
    """Executing the same cached plan twice appends at the same place (execute() truncates back to the encoded
    length first): identical answers, identical cache bytes."""
    cfg, reqs, tok, dec = make(cuda)
    cache = dec.encode_states([r.state for r in reqs], cap=STATE + APPEND)
    a1 = _flat(_decide_cached(dec, reqs, cache))
    k1 = [t.q.clone() for t in cache.k]
    a2 = _flat(_decide_cached(dec, reqs, cache))
    assert all(np.array_equal(x, y) for x, y in zip(a1, a2))
    assert all(torch.equal(x, t.q) for x, t in zip(k1, cache.k))
    assert cache.T == STATE + APPEND


def test_append_prefix_read_paths_identical(cuda):
    """The kept bf16 copy, the per-layer copy made for the pass and the in-kernel dequantisation of the int8 prefix
    give the same answers, bit for bit."""
    cfg, reqs, tok, dec = make(cuda)
    bb = dec.model.backbone
    runs = []
    for mode in ("kept", "jit", "int8"):
        budget0 = bb.materialize_budget
        if mode != "kept":
            bb.materialize_budget = 0
        cache = dec.encode_states([r.state for r in reqs], cap=STATE + APPEND)
        assert (cache.kb is not None) == (mode == "kept")
        bb.materialize_budget = budget0
        bb.jit_min_slots = 0 if mode == "jit" else None
        runs.append(_flat(_decide_cached(dec, reqs, cache)))
        bb.jit_min_slots = 256
    for other in runs[1:]:
        assert all(np.array_equal(x, y) for x, y in zip(runs[0], other))


def test_append_decide_stream_equals_execute(cuda):
    """decide_stream over an encoded cache ((requests, appends) per batch, each batch appending to the encoded
    states afresh) answers as plan + execute does, batch after batch."""
    cfg, reqs, tok, dec = make(cuda)
    cache = dec.encode_states([r.state for r in reqs], room=APPEND)
    want = _flat(_decide_cached(dec, reqs, cache))
    other = syn.decision_requests(5, seed=4, n_requests=N_REQ, vocab=cfg.vocab, state_tokens=STATE,
                                  n_options=OPTIONS, append_tokens=APPEND)[0]
    appends = [[r.append for r in reqs], [r.append for r in other], [r.append for r in reqs]]
    got = [_flat(a) for a, _ in dec.decide_stream(((reqs, ap) for ap in appends), cache=cache)]
    assert len(got) == 3
    for i in (0, 2):
        assert all(np.array_equal(x, y) for x, y in zip(want, got[i]))
    assert not np.array_equal(want[0], got[1][0])        # other records, other answers
