"""od_prefix_attn_noalloc (the split attention with its workspace in the library's static device scratch) against
od_prefix_attn with a caller workspace: identical outputs and LSE on two calls in a row, and an oversize request
rejected on the host. Collected last; passes alone and after the other tests."""
import pytest
import torch

from opendecider_b200 import _lib
from opendecider_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _case(cuda, seed):
    g = syn.gen(seed)
    ac = syn.attn_case(S=2, T=900, rows=3, t=4, Hq=32, Hkv=8, D=128, seed=seed)
    Kq, Vq = ac.Kq.to(cuda), ac.Vq.to(cuda)
    ks, vs = ac.ks.reshape(ac.Kq.shape[:3]).to(cuda), ac.vs.reshape(ac.Kq.shape[:3]).to(cuda)
    Kqn = torch.randn(2, 17, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    Vqn = torch.randn(2, 17, 8, 128, generator=g).to(torch.bfloat16).to(cuda)
    args = dict(Kp=Kq, Vp=Vq, ksc=ks, vsc=vs, row_state=ac.row_state.to(cuda),
                p_lo=torch.tensor([0, 41], dtype=torch.int32, device=cuda), Kq=Kqn, Vq=Vqn,
                row_q=torch.tensor([0, 1, 1, 0, 1, 0], dtype=torch.int32, device=cuda),
                q_len=torch.tensor([17, 6], dtype=torch.int32, device=cuda), want_lse=True)
    return ac.q.to(cuda), ac.k.to(cuda), ac.v.to(cuda), args


def test_no_alloc_equals_workspace_variant_twice(cuda):
    for seed in (41, 42):                                   # two calls in a row, different inputs
        q, k, v, args = _case(cuda, seed)
        o_ws, l_ws = _lib.prefix_attn(q, k, v, 128 ** -0.5, nsplit=3, **args)
        o_na, l_na = _lib.prefix_attn_noalloc(q, k, v, 128 ** -0.5, nsplit=3, **args)
        torch.cuda.synchronize()
        assert _lib.device_error(cuda) == 0
        assert torch.equal(o_ws, o_na), seed
        assert torch.equal(l_ws, l_na), seed


def test_no_alloc_without_split_needs_no_scratch(cuda):
    q, k, v, args = _case(cuda, 43)
    o1, l1 = _lib.prefix_attn(q, k, v, 128 ** -0.5, nsplit=1, **args)
    o2, l2 = _lib.prefix_attn_noalloc(q, k, v, 128 ** -0.5, nsplit=1, **args)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_no_alloc_empty_problem(cuda):
    """No rows (or no tokens) with a split requested: both variants return without a launch and without scratch."""
    q, k, v, args = _case(cuda, 45)
    no_rows = (q[:0], k[:0], v[:0])
    no_tokens = (q[:, :0].contiguous(), k[:, :0].contiguous(), v[:, :0].contiguous())
    for qe, ke, ve in (no_rows, no_tokens):
        o1, l1 = _lib.prefix_attn(qe, ke, ve, 128 ** -0.5, nsplit=3, **args)
        o2, l2 = _lib.prefix_attn_noalloc(qe, ke, ve, 128 ** -0.5, nsplit=3, **args)
        assert o1.numel() == o2.numel() == 0 and l1.numel() == l2.numel() == 0
    torch.cuda.synchronize()
    assert _lib.device_error(cuda) == 0


def test_no_alloc_rejects_oversize_scratch(cuda):
    """64 splits of 6 rows x 4 tokens x 32 heads x 129 floats need 25 MB > the 16 MiB scratch: refused on the
    host, nothing launched."""
    q, k, v, args = _case(cuda, 44)
    with pytest.raises(_lib.ODError, match="static scratch"):
        _lib.prefix_attn_noalloc(q, k, v, 128 ** -0.5, nsplit=64, **args)
