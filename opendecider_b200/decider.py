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
from .staging import Staging

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
        self.staging = Staging(model.backbone.device)
        self._graphs = {}                         # execute_graph: plan layout -> (CUDA graph, its outputs)
        self._graph_pool = None
        if torch.device(model.backbone.device).type == "cuda":
            self._graph_pool = torch.cuda.graph_pool_handle()

    def _with_none(self, q: Question) -> Question:
        """Copy of q with `none` appended, unless at the 255-option cap (decider.py:296-303)."""
        if getattr(q, "none", None) is False or len(q.options) >= MAX_OPTIONS:
            return q
        q2 = copy.copy(q)
        q2.options = list(q.options) + [self.none_text]
        q2.none_col = len(q.options)
        return q2

    def encode_states(self, states, cap: int | None = None, room: int = 0) -> KVCache:
        """The batched state pass: state_text() of every request, tokenised, one left-padded pass (in state chunks
        for long states). cap (total token capacity) or room (tokens beyond the encoded length): space for appended
        tokens (decide with `cache=` and `appends=`)."""
        st = self._plan_states(states)
        st["cap"] = max(cap or 0, st["T"] + room)
        return self.model.backbone.run_state(st)

    def _plan_states(self, states, up=None) -> dict:
        texts = [state_text(s) for s in states]
        seqs = self.model.tok(texts, add_special_tokens=False)["input_ids"]
        return self.model.backbone.plan_state(seqs, up)

    def plan_questions(self, requests) -> dict:
        """The host-only part of a plan (the question list and owners) for building answers from gathered results."""
        batch, owner = [], []
        for i, r in enumerate(requests):
            for q in r.questions:
                q2 = copy.copy(q)
                q2.state_idx = i
                q2.name = f"{i}\x1f{q.name}"
                batch.append(self._with_none(q2) if self.none_text else q2)
                owner.append(i)
        return {"questions": batch, "owner": owner, "n_requests": len(requests)}

    def plan(self, requests, cache: KVCache | None = None, appends=None) -> dict:
        """Everything host-side of one decide_many call (tokenisation, layouts, readout constants), staged in one
        pinned buffer and uploaded by one copy. The plan's device views stay valid until the next plan().
        With `cache` (row i = request i's encoded state, encode_states) the state pass is skipped; `appends` (one text
        per request, equal token counts) are first appended to the states - PrefixCache.encode's continuation of a
        cached state (state_cache.py:116-158) for the whole batch - and the questions read the extended states."""
        self.staging.begin()
        up = self.staging.put
        if cache is None:
            st = self._plan_states([r.state for r in requests], up)
        else:
            assert cache.S == len(requests), "one cached state per request"
            T0, lens0 = cache.enc_T, list(cache.enc_lens)        # appends of earlier calls are not kept
            app, n = None, 0
            if appends is not None:
                seqs = self.model.tok(list(appends), add_special_tokens=False)["input_ids"]
                n = len(seqs[0])
                assert all(len(q) == n for q in seqs), "appends of one batch have equal token counts"
                assert T0 + n <= cache.capacity, "the cache has no room for the appended tokens (encode_states cap)"
                app = up(torch.tensor(seqs, dtype=torch.long))
            st = {"cached": True, "T0": T0, "lens0": lens0, "append": app, "T": T0 + n, "lens": [l + n for l in lens0]}
        batch, owner = [], []
        for i, r in enumerate(requests):
            for q in r.questions:
                q2 = copy.copy(q)
                q2.state_idx = i
                q2.name = f"{i}\x1f{q.name}"
                batch.append(self._with_none(q2) if self.none_text else q2)
                owner.append(i)
        T = up(torch.tensor([self.temperature_by_type.get(q.type, self.temperature) for q in batch],
                            dtype=torch.float32))
        nc = up(torch.tensor([getattr(q, "none_col", -1) for q in batch], dtype=torch.int32))
        mplan = self.model.plan(batch, st["T"], st["lens"], up)
        h2d = self.staging.commit()
        return {"state": st, "model": mplan, "questions": batch, "owner": owner, "n_requests": len(requests),
                "T": T, "none_col": nc, "h2d_bytes": h2d}

    def execute(self, plan: dict, cache: KVCache | None = None):
        """The device work of one call: state pass, row passes, trunk, od_readout. Returns device tensors
        (probs (N, K) fp32, renorm (N, K) fp64, p_none (N,) fp32) and the cache."""
        st = plan["state"]
        if st.get("cached"):
            assert cache is not None, "the plan reads an encoded cache: pass it to execute()"
            cache.truncate(st["T0"], st["lens0"])         # a replayed plan appends at the same place again
            if st["append"] is not None:
                self.model.backbone.run_append(st["append"], cache)
        else:
            cache = self.model.backbone.run_state(st, cache)
        logits, opt_mask = self.model.execute(plan["model"], cache)
        probs = _lib.readout(logits.contiguous(), plan["T"], opt_mask.to(torch.uint8), none_col=plan["none_col"])
        return probs, cache

    def execute_graph(self, plan: dict, cache: KVCache | None = None):
        """execute() as ONE CUDA graph per plan layout: the first call with a layout runs execute() eagerly (setting
        up the kernels' one-time attributes and the cache), then captures it; later calls with the same layout - the
        same shapes and the same staging offsets, so a new batch of the same structure whose plan has just been
        staged - replay it. Every kernel of the state pass, the row passes, the trunk and the readout is in the graph;
        the plan's inputs live in the staging arena's device buffer, whose addresses the graph captured, and the
        outputs in the graph's memory pool (read them before the next replay). The cache must be the one of the
        capture (the plan layout includes its buffers)."""
        if cache is None:
            probs, cache = self.execute(plan, cache)       # allocates the cache outside any graph
            torch.cuda.synchronize(self.model.backbone.device)
        key = (_layout(plan), _layout(cache))
        hit = self._graphs.get(key)
        if hit is None:
            dev = self.model.backbone.device
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                self.execute(plan, cache)                  # warm-up: one-time kernel attributes, allocator pools
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self._graph_pool):
                out, c2 = self.execute(plan, cache)
            assert c2 is cache, "the captured pass must write the given cache"
            hit = self._graphs[key] = (graph, out)
        graph, out = hit
        graph.replay()
        return out, cache

    def probs(self, questions, cache: KVCache):
        """Decider._probs (decider.py:236-284) without calibration profiles / sampler for questions reading
        `cache`: logits / T -> softmax * mask, caller-option renormalisation (fp64) and P(none) in od_readout."""
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

    def answers(self, plan: dict, probs) -> list:
        """Host answers from the device results (one device->host read of probs, renorm and P(none))."""
        got = self._answers(plan["questions"], *probs)
        out = [{} for _ in range(plan["n_requests"])]
        for q, i in zip(plan["questions"], plan["owner"]):
            out[i][q.name.split("\x1f", 1)[1]] = got[q.name]
        return out

    def decide_many(self, requests) -> list:
        """Independent requests in one batch: ONE state pass over all states and ONE row pass over all questions,
        each question reading its own request's state (decider.py:438-484). Returns per request {name: answer}
        (no requests: []; requests without questions: {} each, and no backbone pass)."""
        if not requests or not any(r.questions for r in requests):
            return [{} for _ in requests]
        plan = self.plan(requests)
        probs, _ = self.execute(plan)
        return self.answers(plan, probs)

    def decide_stream(self, batches, gather=None, cache: KVCache | None = None):
        """decide_many over a sequence of request batches, pipelined: the read-back of batch b's results is enqueued
        right after its kernels, batch b+1 is planned on the host and its device work enqueued, and only then are
        b's results awaited, so the GPU runs batch after batch without waiting for the host. `gather(probs)`
        (optional) runs on the device after a batch's kernels, in stream order (e.g. the data-parallel all-gather of
        the probabilities), and its result is read back with the answers. Yields (answers, gathered or None) per
        batch, in order. The KV cache allocation is reused from batch to batch. With `cache`, every batch is a
        (requests, appends) pair over that cache's encoded states (see plan())."""
        pending, fixed = None, cache is not None
        for item in batches:
            plan = self.plan(item[0], cache=cache, appends=item[1]) if fixed else self.plan(item)
            probs, cache = self.execute(plan, cache)
            dev = list(probs) + ([gather(probs)] if gather is not None else [])
            host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dev]
            for h, d in zip(host, dev):
                h.copy_(d, non_blocking=True)
            done = torch.cuda.Event()
            done.record(torch.cuda.current_stream(self.model.backbone.device))
            self.last_io = {"h2d_bytes": plan["h2d_bytes"], "d2h_bytes": sum(h.numel() * h.element_size() for h in host)}
            if pending is not None:
                yield self._finish(*pending)
            pending = (plan, host, done, gather is not None)
        if pending is not None:
            yield self._finish(*pending)

    def _finish(self, plan: dict, host: list, done, gathered: bool):
        done.synchronize()
        return self.answers(plan, host[:3]), (host[3] if gathered else None)


def _layout(x):
    """Hashable layout of a plan or cache: device tensors by (address, shape, dtype), host tensors and scalars by
    value, host-only objects (questions, owners) skipped. Two plans with the same layout launch the same kernels on
    the same buffers."""
    import dataclasses
    if isinstance(x, torch.Tensor):
        if x.device.type == "cpu":                       # host-side plan data: its values shape the launches
            return ("C", tuple(x.reshape(-1).tolist()), tuple(x.shape), str(x.dtype))
        return ("T", x.data_ptr(), tuple(x.shape), str(x.dtype), x.device.type)
    if isinstance(x, (int, float, bool, str, type(None))):
        return x
    if isinstance(x, dict):
        return tuple((k, _layout(v)) for k, v in x.items() if k not in ("questions", "owner", "h2d_bytes"))
    if isinstance(x, (list, tuple)):
        return tuple(_layout(v) for v in x)
    if dataclasses.is_dataclass(x):
        # a pass's cache and question-level K/V are bound when the pass runs (run_rows): not part of the plan's layout
        skip = ("cache", "qkv_prefix") if type(x).__name__ == "PassSpec" else ()
        return (type(x).__name__,) + tuple(_layout(getattr(x, f.name)) for f in dataclasses.fields(x)
                                           if f.name not in skip)
    return ("obj", type(x).__name__)
