"""The trunk's host-side layout (opendecider_b200.v3.trunk_plan): the forms the kernels read - flat destination rows,
int32 option ids with -1 padding, flat positions, real token counts per question - describe the same layout as the
2-D tensors the CPU oracle reads (oracle/trunk.py), on ragged questions; and V3Trunk refuses a CPU device (the
product has no CPU path)."""
import pytest
import torch

from opendecider_b200 import _lib
from opendecider_b200.v3 import TrunkConfig, V3Trunk, trunk_plan, trunk_state_dict


def _case(seed=0, n=9):
    g = torch.Generator().manual_seed(seed)
    n_opt = torch.randint(1, 7, (n,), generator=g)
    o_lens = torch.randint(1, 5, (int(n_opt.sum()),), generator=g)
    q_lens = torch.randint(1, 30, (n,), generator=g)
    state_lens = torch.randint(0, 5000, (n,), generator=g)
    return q_lens, o_lens, n_opt, state_lens


def test_trunk_plan_kernel_forms_match_the_layout():
    q_lens, o_lens, n_opt, state_lens = _case()
    p = trunk_plan(q_lens, o_lens, n_opt, state_lens, lambda x: x)
    N, K, P, Tc = p["N"], p["K"], p["P"], p["Tc"]
    row, col = p["rc"]
    assert torch.equal(p["rc_flat"], row * P + col)
    qrow, qcol = p["qrc"]
    assert torch.equal(p["qrc_flat"], qrow * Tc + qcol)
    assert torch.equal(p["gid32"].long(), p["opt_id"]) and p["gid32"].dtype == torch.int32
    assert torch.equal(p["opos32"].long(), p["opos"].reshape(-1))
    assert torch.equal(p["cpos32"].long(), p["cpos"].reshape(-1))
    assert torch.equal(p["cgid32"] < 0, p["c_pad"])
    # real tokens are a prefix of each row: option tokens, question tokens, options
    assert torch.equal(p["olen32"].long(), (p["opt_id"] >= 0).sum(1))
    for b in range(N):
        assert bool((p["opt_id"][b, : int(p["olen32"][b])] >= 0).all())
        assert bool((~p["c_pad"][b, : int(p["qlen32"][b])]).all()) and bool(p["c_pad"][b, int(p["qlen32"][b]):].all())
    assert torch.equal(p["nopt32"].long(), n_opt) and K == int(n_opt.max())
    assert torch.equal(p["opt_mask"].sum(1), n_opt)
    # every option's tokens carry its index and positions 0..len-1
    starts = torch.cumsum(n_opt, 0) - n_opt
    for b in range(N):
        for k in range(int(n_opt[b])):
            sel = p["opt_id"][b] == k
            assert int(sel.sum()) == int(o_lens[starts[b] + k])
            assert torch.equal(p["opos"][b][sel], torch.arange(int(sel.sum())))


def test_v3trunk_has_no_cpu_path():
    tc = TrunkConfig(d_feat=64, n_feat_layers=1, d_model=32, n_heads=2, decision_layers=1)
    with pytest.raises(_lib.ODError):
        V3Trunk(tc, trunk_state_dict(tc, seed=0), "cpu")


def test_trunk_seam_reads_every_trunk_parameter():
    """prepare_b200_'s trunk seam takes a reference model's trunk entries by name prefix: every parameter V3Trunk
    reads (the reference V3's names, with and without the LM feature) matches one, and the backbone's do not."""
    from opendecider_b200.integrate import _TRUNK_PREFIXES
    for lm in (False, True):
        tc = TrunkConfig(d_feat=64, n_feat_layers=3, d_model=32, n_heads=2, decision_layers=2, lm_feature=lm)
        assert [k for k in trunk_state_dict(tc) if not k.startswith(_TRUNK_PREFIXES)] == []
    assert not any(k.startswith(_TRUNK_PREFIXES) for k in ("backbone.lm.layers.0.self_attn.q_proj.qweight",
                                                            "vera.b.0", "context_layers.0.n1.g", "slots.emb"))
