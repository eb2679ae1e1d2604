"""Decision orchestration on B200: requests -> one left-padded state pass -> one row pass over every question ->
the option/`none` readout (od_readout). Mirrors Decider.decide_many / _answer_batch / _probs of the reference
(src/opendecider/decider.py:236-361, 438-484) for atomic questions.

Out of this path (the reference's host-side API layer, unchanged semantics not rebuilt here): dependency waves and
chaining, composite questions, calibration profiles, conformal sets, the sampler (k > 1) and the two-stage path for
more than 255 options.
"""
from __future__ import annotations

import copy
import math
import os

import torch

from . import _lib
from .backbone import KVCache
from .batching import MAX_OPTIONS, Question, state_text

# option rows per call from which the question cache is used (decider.py:85-88, keyed by backbone hidden size)
QCACHE_MIN_ROWS = {2048: 64, 4096: 12}


class Decider:
    def __init__(self, model, temperature: float = 1.0, temperature_by_type: dict | None = None,
                 none_text: str | None = None):
        self.model = model
        self.temperature = temperature
        self.temperature_by_type = temperature_by_type or {}
        # the explicit `none` option appended as text to every question (decider.py:133-135)
        self.none_text = os.environ.get("OPENDECIDER_NONE_TEXT", "none of the above") if none_text is None \
            else none_text

    def _with_none(self, q: Question) -> Question:
        """Copy of q with `none` appended, unless at the 255-option cap (decider.py:296-303)."""
        if getattr(q, "none", None) is False or len(q.options) >= MAX_OPTIONS:
            return q
        q2 = copy.copy(q)
        q2.options = list(q.options) + [self.none_text]
        q2.none_col = len(q.options)
        return q2

    def encode_states(self, states) -> KVCache:
        """The batched state pass: state_text() of every request, tokenised, one left-padded pass."""
        texts = [state_text(s) for s in states]
        seqs = self.model.tok(texts, add_special_tokens=False)["input_ids"]
        return self.model.backbone.prefix_cache_batch(seqs)

    def probs(self, questions, cache: KVCache):
        """Decider._probs (decider.py:236-284) without calibration profiles / sampler: logits / T -> softmax * mask,
        the caller-option renormalisation in fp64 and P(none), all in od_readout. Returns device tensors
        (probs (N, K) fp32, renorm (N, K) fp64, p_none (N,) fp32)."""
        logits, opt_mask = self.model.run(questions, cache)
        dev = logits.device
        T = torch.tensor([self.temperature_by_type.get(q.type, self.temperature) for q in questions],
                         dtype=torch.float32).to(dev, non_blocking=True)
        nc = torch.tensor([getattr(q, "none_col", -1) for q in questions], dtype=torch.int32).to(dev,
                                                                                               non_blocking=True)
        return _lib.readout(logits.contiguous(), T, opt_mask.to(torch.uint8), none_col=nc)

    def _answers(self, questions, probs, renorm, p_none) -> dict:
        """Per-question answers (decider.py:330-358): renormalised probabilities over the caller's options,
        value, Jev-style confidence, P(none)."""
        p, ren, pn = probs.cpu(), renorm.cpu(), p_none.cpu()
        out = {}
        for i, q in enumerate(questions):
            K = getattr(q, "none_col", len(q.options))
            pl = ren[i, :K].tolist()
            names = getattr(q, "names", None) or q.options[:K]
            pmax = max(pl)
            a = {"value": names[max(range(K), key=pl.__getitem__)],
                 "confidence": max(0.0, min(1.0, (K * pmax - 1) / (K - 1))) if K > 1 else 1.0,
                 "probs": dict(zip(names, pl)), "probs_list": pl}
            if hasattr(q, "none_col"):
                a["none"] = float(pn[i])
                if a["none"] > float(p[i, :K].max()):
                    a["value"] = "none"
            if q.type == "noul":
                a["p_yes"] = pl[0]
            if q.type == "score":
                a["expected_index"] = sum(k * v for k, v in enumerate(pl))
            out[q.name] = a
        return out

    def decide_many(self, requests) -> list:
        """Independent requests in one batch: ONE state pass over all states and ONE row pass over all questions,
        each question reading its own request's state (decider.py:438-484). Returns per request {name: answer}."""
        cache = self.encode_states([r.state for r in requests])
        batch, owner = [], []
        for i, r in enumerate(requests):
            for q in r.questions:
                q2 = copy.copy(q)
                q2.state_idx = i
                q2.name = f"{i}\x1f{q.name}"
                batch.append(self._with_none(q2) if self.none_text else q2)
                owner.append(i)
        probs, renorm, p_none = self.probs(batch, cache)
        got = self._answers(batch, probs, renorm, p_none)
        out = [{} for _ in requests]
        for q, i in zip(batch, owner):
            out[i][q.name.split("\x1f", 1)[1]] = got[q.name]
        return out
