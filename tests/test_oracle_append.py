"""The oracle's continuation of cached states (OracleDecision.append_pass) pinned to the reference's own PrefixCache
(tests/golden/append_config5.npz, made by tests/golden/make_golden_append.py): 2 requests, 96-token states, 24
appended ids, the tiny backbone of the e2e fixture.

Everything is compared byte for byte: the oracle's attention over the restored prefix is the reference's own CPU
call (torch's scaled_dot_product_attention, as transformers makes it), so the chained layers' K/V, the snapshots and
the packed cache equal the reference's exactly in every layer, on the machine that made the fixture."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from make_golden_append import APPEND, N_REQ, OPTIONS, STATE  # noqa: E402
from make_golden_e2e import FEATURE_LAYERS  # noqa: E402

from oracle import ops  # noqa: E402
from oracle.model import BF, OracleDecision  # noqa: E402
from opendecider_b200 import synthetic as syn  # noqa: E402
from opendecider_b200.backbone import DecoderConfig, synthetic_weights  # noqa: E402

@pytest.fixture(scope="module")
def setup():
    cfg = DecoderConfig.tiny(feature_layers=tuple(FEATURE_LAYERS))
    reqs, tok = syn.decision_requests(5, seed=3, n_requests=N_REQ, vocab=cfg.vocab, state_tokens=STATE,
                                      n_options=OPTIONS, append_tokens=APPEND)
    g = np.load(os.path.join(HERE, "golden", "append_config5.npz"))
    od = OracleDecision(cfg, synthetic_weights(cfg, seed=0), None, tok, {}, 1.0)
    runs = []
    for req in reqs:
        pre = od.state_pass([req.state])
        runs.append(od.append_pass(pre, [req.append]))
    return cfg, reqs, tok, g, od, runs


def _bits(t):
    return t.contiguous().view(torch.int16).numpy()


def test_appended_ids_are_the_golden_inputs(setup):
    cfg, reqs, tok, g, od, runs = setup
    for req in reqs:
        assert len(tok([req.append], add_special_tokens=False)["input_ids"][0]) == APPEND


def test_layer0_snapshot_bit_exact(setup):
    """The first layer's appended K/V (positions 96..119) as the reference's _take quantises them."""
    cfg, reqs, tok, g, od, runs = setup
    for r, (_, snaps, _) in enumerate(runs):
        for a, (q8, sc) in zip("kv", snaps[0]):
            np.testing.assert_array_equal(q8[0].numpy(), g[f"snap.{r}.0.{a}.q"])
            np.testing.assert_array_equal(_bits(sc[0]), g[f"snap.{r}.0.{a}.s"])


def test_every_layer_kv_write_bit_exact_on_reference_input(setup):
    """Each layer's K/V write given the hidden state the reference fed that layer: projections, norms, RoPE at the
    continued positions and the snapshot quantisation, byte for byte, in all layers."""
    cfg, reqs, tok, g, od, runs = setup
    pos = (STATE + torch.arange(APPEND))[None]

    def no_attend(i, q, k, v):
        return torch.zeros(q.shape[0], q.shape[1], q.shape[2] * q.shape[3], dtype=BF)

    for r in range(N_REQ):
        for li in range(cfg.layers):
            x = torch.from_numpy(g[f"xin.{r}.{li}"]).view(BF)[None]
            _, k, v = od.dec.layer(li, x, pos, no_attend)
            for a, t in (("k", k), ("v", v)):
                q8, sc, _ = ops.quantize_rows(t[0].transpose(0, 1).float().numpy(), "bf16")
                np.testing.assert_array_equal(q8, g[f"snap.{r}.{li}.{a}.q"], err_msg=f"req {r} layer {li} {a}")
                np.testing.assert_array_equal(_bits(torch.from_numpy(sc[..., 0]).to(BF)), g[f"snap.{r}.{li}.{a}.s"])


def test_chained_layers_bit_exact(setup):
    """Every layer's appended K/V after the chained continuation (each layer's attention reads the restored prefix
    and the earlier appended tokens): the snapshot bytes and scales and the packed cache, equal to the reference's."""
    cfg, reqs, tok, g, od, runs = setup
    for r, (_, snaps, packs) in enumerate(runs):
        for li in range(cfg.layers):
            for ai, a in enumerate("kv"):
                for name, (q8, sc) in (("snap", snaps[li][ai]), ("pack", packs[li][ai])):
                    np.testing.assert_array_equal(q8[0].numpy(), g[f"{name}.{r}.{li}.{a}.q"],
                                                  err_msg=f"{name} req {r} layer {li} {a}")
                    np.testing.assert_array_equal(_bits(sc[0]), g[f"{name}.{r}.{li}.{a}.s"])


def test_pack_layer0_bit_exact(setup):
    """PackedCache.pack re-quantises the materialised prefix with the new K/V: layer 0 (no attention upstream of
    either part) equals the reference byte for byte, prefix and appended slice."""
    cfg, reqs, tok, g, od, runs = setup
    for r, (_, _, packs) in enumerate(runs):
        for a, (q8, sc) in zip("kv", packs[0]):
            np.testing.assert_array_equal(q8[0].numpy(), g[f"pack.{r}.0.{a}.q"])
            np.testing.assert_array_equal(_bits(sc[0]), g[f"pack.{r}.0.{a}.s"])
