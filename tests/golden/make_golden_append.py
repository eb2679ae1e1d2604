"""Golden K/V of a cached-state continuation (BASELINE config 5 at reduced scale), produced by the REFERENCE's own
PrefixCache (src/opendecider/state_cache.py:116-158) on CPU in bf16.

Set-up: the reference backbone of make_golden_e2e.py (tiny all-attention Qwen3.5, synthetic weights seed 0, the
reference's int8 weight / KV quantisers, the W8A8 arithmetic at the Int8Linear._fused seam, the word-level
SyntheticTokenizer). For each of 2 requests of decision_requests(5, ...) (96-token states, 24 appended ids):
  1. PrefixCache.encode([state_text(state)], [])                       -> snapshot of the state (int8 K/V)
  2. PrefixCache.encode([state_text(state), append_text], [])          -> resumes from that snapshot: the appended
     ids are prefilled against the restored (materialised) prefix with positions continuing at 96, their K/V are
     quantised into the next snapshot, and the whole cache is packed (PackedCache.pack re-quantises the prefix).
Writes tests/golden/append_config5.npz: per request and layer, the appended tokens' snapshot quantisation
(`snap.{r}.{layer}.{k|v}.q` int8 (Hkv, 24, D), `.s` bf16 bits (Hkv, 24)), the final packed cache
(`pack.{r}.{layer}.{k|v}.q` (Hkv, 120, D), `.s` (Hkv, 120)) and the hidden state entering each decoder layer for
the appended tokens in the continuation pass (`xin.{r}.{layer}` bf16 bits (24, hidden)), so that each layer's K/V
write can be checked on the reference's own input.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden_e2e import FEATURE_LAYERS, build_reference, use_reference  # noqa: E402

from opendecider_b200 import synthetic as syn  # noqa: E402
from opendecider_b200.backbone import DecoderConfig  # noqa: E402
from opendecider_b200.batching import state_text  # noqa: E402

N_REQ, STATE, APPEND, OPTIONS = 2, 96, 24, 20


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy()


def main():
    use_reference()
    from opendecider.state_cache import PrefixCache
    torch.manual_seed(0)
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    reqs, tok = syn.decision_requests(5, seed=3, n_requests=N_REQ, vocab=cfg.vocab, state_tokens=STATE,
                                      n_options=OPTIONS, append_tokens=APPEND)
    bb = build_reference(cfg, tok)
    out = {}
    for r, req in enumerate(reqs):
        pc = PrefixCache(bb, max_bytes=1 << 30)
        s_text = state_text(req.state)
        xin = {}
        hooks = [layer.register_forward_pre_hook(
            lambda m, args, kwargs, li=li: xin.__setitem__(li, (args[0] if args else kwargs["hidden_states"]).clone()),
            with_kwargs=True) for li, layer in enumerate(bb.lm.layers)]
        with torch.no_grad():
            pc.encode([s_text], [])
            xin.clear()
            packed, mask, n_cached = pc.encode([s_text, req.append], [])
        for h in hooks:
            h.remove()
        assert n_cached == STATE and mask.shape[1] == STATE + APPEND, (n_cached, mask.shape)
        snap = pc.snaps[list(pc.snaps)[-1]]
        assert snap.n_tokens == STATE + APPEND
        for li in range(cfg.layers):
            assert xin[li].shape == (1, APPEND, cfg.hidden), xin[li].shape
            out[f"xin.{r}.{li}"] = bits(xin[li][0])
            for a, name in (("k", "keys"), ("v", "values")):
                sq = snap.kv[(li, name)]
                out[f"snap.{r}.{li}.{a}.q"] = sq.q[0].numpy()
                out[f"snap.{r}.{li}.{a}.s"] = bits(sq.scale[0, ..., 0])
                pq = packed.tensors[(li, name, None)]
                out[f"pack.{r}.{li}.{a}.q"] = pq.q[0].numpy()
                out[f"pack.{r}.{li}.{a}.s"] = bits(pq.scale[0, ..., 0])
    np.savez_compressed(os.path.join(HERE, "append_config5.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
