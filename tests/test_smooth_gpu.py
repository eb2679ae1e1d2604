"""SmoothQuant (the reference's a8w8sq path: smooth_a8w8_ + SmoothedLinear, quant.py:317-350) through the B200
decision forward, on BASELINE config 1 with scales calibrated by the reference's own procedure
(tests/golden/smooth_config1.npz, made by tests/golden/make_golden_smooth.py):

  - per-linear vectors (q, k, v, gate, up each their own, as the reference calibrates them): the separate
    quantisations and GEMMs (od_gemm_w8a8_ld into the stacked q/k/v output, two MLP GEMMs + od_swiglu_quant);
  - one shared vector per input (q/k/v, gate/up): the fused GEMMs with the multiply inside the quantiser.

Checks: the state pass's layer-0 K/V (embedding, RMSNorm, the smoothed k/v projections and the cache quantisation)
equal the oracle's except where RMSNorm's fp32 sum of squares, reduced in another order, flips a bf16 value by one
ulp (a few elements in 10^5) - a wrong or missing smoothing changes nearly all of them; the decisions are within 1e-3
of the reference's (per-linear) and of the oracle's (shared)."""
import numpy as np
import pytest
import torch

from oracle import ops
from oracle.model import OracleDecision
from oracle.trunk import OracleTrunk
from opendecider_b200 import synthetic as syn
from opendecider_b200.backbone import Backbone, DecoderConfig, synthetic_weights
from opendecider_b200.decider import Decider
from opendecider_b200.v3 import TrunkConfig, V3Model, V3Trunk, trunk_state_dict

pytestmark = pytest.mark.gpu

FEATURE_LAYERS = (1, 3, "final")
TRUNK = dict(d_model=64, n_heads=4, decision_layers=2)
TEMPS = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}
TEMPERATURE = 1.419344425201416


def _scales(shared: bool) -> dict:
    g = np.load("tests/golden/smooth_config1.npz")
    sc = {k[len("scale."):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("scale.")}
    if shared:                                        # one vector per input: q/k/v share q's, gate/up share gate's
        for i in range(4):
            p = f"{i}."
            for n in ("self_attn.k_proj", "self_attn.v_proj"):
                sc[p + n] = sc[p + "self_attn.q_proj"]
            sc[p + "mlp.up_proj"] = sc[p + "mlp.gate_proj"]
    return sc


def _deciders(cuda, smooth):
    cfg = DecoderConfig.tiny(feature_layers=FEATURE_LAYERS)
    sd = synthetic_weights(cfg, seed=0)
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(FEATURE_LAYERS), **TRUNK)
    reqs, tok = syn.decision_requests(1, seed=0)
    bb = Backbone.from_float_weights(cfg, sd, cuda, smooth=smooth)
    dec = Decider(V3Model(bb, V3Trunk(tc, trunk_state_dict(tc, seed=0), cuda), tok, qcache_min_rows=32),
                  TEMPERATURE, TEMPS)
    od = OracleDecision(cfg, sd, OracleTrunk(tc, trunk_state_dict(tc, seed=0)), tok, TEMPS, TEMPERATURE,
                        qcache_min_rows=32, smooth=smooth)
    return dec, od, reqs


def _collect(ans):
    p = np.array([a["q0"]["probs_list"] for a in ans])
    return p, np.array([a["q0"]["none"] for a in ans])


@pytest.mark.parametrize("shared", [False, True])
def test_smoothquant_layer0_kv_bytes_and_decisions(cuda, shared):
    smooth = _scales(shared)
    dec, od, reqs = _deciders(cuda, smooth)
    bb = dec.model.backbone
    L0 = bb.layers[0]
    assert L0.sq is not None and L0.sq.qkv_shared == shared and L0.sq.gu_shared == shared
    assert (L0.gate_up is None) == (not shared)
    # layer-0 K/V of the state pass vs the oracle's, dequantised exactly as materialize() does
    cache = dec.encode_states([r.state for r in reqs])
    ocache, _, T, _ = od.state_pass([r.state for r in reqs])
    for a, ref in ((cache.k[0], ocache[0][0]), (cache.v[0], ocache[0][1])):
        got = ops.materialize_int8(a.q[:, :, :T].cpu(), a.scale[:, :, :T, None].cpu())
        differ = (got != ref).float().mean().item()
        assert differ < 1e-3, differ
        assert (got.float() - ref.float()).abs().max() <= 0.05 * ref.float().abs().max()
    p, none = _collect(dec.decide_many(reqs))
    if shared:
        _, ren, pn, _ = od.decide(reqs)
        want, want_none = ren[:, : p.shape[1]], pn
    else:
        g = np.load("tests/golden/smooth_config1.npz")
        want, want_none = g["probs"], g["none"]
    assert np.abs(p - want).max() < 1e-3, np.abs(p - want).max()
    assert np.abs(none - want_none).max() < 1e-3


@pytest.mark.parametrize("M", [300, 1500])
def test_gemm_ld_and_narrow_n(cuda, M):
    """od_gemm_w8a8_ld writes column ranges of a wider output, and N = 128, 96 or 32 (a last tile narrower than 256
    columns, the tiny model's separate k / v projections): the same bytes as one full-width GEMM, on the single-CTA
    (M = 300) and the CTA-pair (M = 1500) forms."""
    from opendecider_b200 import _lib
    gc = syn.gemm_case(M=M, N=512, K=256, seed=4)
    xq, sx = _lib.quant_rows(gc.x.to(cuda), scale_dtype=torch.float32)
    W, sw = gc.qweight.to(cuda), gc.wscale.to(cuda).view(-1)
    full = _lib.gemm_w8a8(xq, sx.view(-1), W, sw, _lib.OD_EPI_BF16)
    wide = torch.zeros(M, 640, dtype=torch.bfloat16, device=cuda)
    for a, n in ((0, 256), (256, 128), (384, 96), (480, 32)):
        _lib.gemm_w8a8(xq, sx.view(-1), W[a:a + n], sw[a:a + n], _lib.OD_EPI_BF16, out=wide[:, a:a + n])
    assert torch.equal(wide[:, :512], full)
    assert not wide[:, 512:].any()                   # nothing written past the column ranges
    i32 = _lib.gemm_w8a8(xq, None, W[:96], None, _lib.OD_EPI_INT32)
    assert torch.equal(i32.cpu(), torch.from_numpy(ops.gemm_i32(xq.cpu().numpy(), gc.qweight[:96].numpy())))
    torch.cuda.synchronize()
    assert _lib.device_error(cuda) == 0
