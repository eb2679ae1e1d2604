"""Generate the golden fixtures of tests/golden/ by running the REFERENCE implementation (OpenDecider's own
src/opendecider code and the transformers Qwen3.5 modules it calls) on seeded inputs from opendecider_b200.synthetic.

Run in a container that has the reference checked out (it is not needed anywhere else):
    OPENDECIDER_REF=/path/to/reference/src python tests/golden/make_golden.py

Writes tests/golden/ops.npz. Inputs are NOT stored: tests regenerate them from the same seeds and check a digest.
bf16/fp16 tensors are stored as their raw 16-bit patterns (uint16/int16 views).
"""
from __future__ import annotations

import hashlib
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
if __name__ == "__main__":
    if not os.environ.get("OPENDECIDER_REF"):     # the reference's src/ directory (this generator imports it)
        sys.exit("set OPENDECIDER_REF to the reference checkout's src/ directory")
    sys.path.insert(0, os.environ["OPENDECIDER_REF"])

from opendecider_b200 import synthetic as syn  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy()
    return t.contiguous().numpy()


def digest(*ts: torch.Tensor) -> np.ndarray:
    h = hashlib.sha256()
    for t in ts:
        h.update(bits(t).tobytes())
    return np.frombuffer(h.digest()[:8], dtype=np.uint8).copy()


def main() -> None:
    import torch.nn as nn
    from opendecider.quant import Int8Embedding, Int8Linear, Int8Tensor, materialize
    from opendecider.prefix_attn import _split_attention
    from opendecider.decider import Decider, _normalize
    from opendecider.batching import Question
    from opendecider.models import DecisionOutput
    from opendecider.sampler import SamplerConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5RMSNorm, apply_rotary_pos_emb

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out: dict[str, np.ndarray] = {}

    # ---- A1 / A5: Int8Linear weight quantiser and Int8Tensor.quantize of bf16 / fp16 / fp32 activations
    gc = syn.gemm_case(M=64, N=256, K=512, seed=1)
    lin = nn.Linear(512, 256, bias=False)
    lin.weight.data = gc.w.clone()
    il = Int8Linear(lin)
    out["gemm.digest"] = digest(gc.x, gc.w)
    out["gemm.qweight"] = bits(il.qweight)
    out["gemm.wscale"] = bits(il.scale)
    for name, x in (("bf16", gc.x), ("f16", gc.x.float().to(torch.float16)), ("f32", gc.x.float())):
        it = Int8Tensor.quantize(x)
        out[f"quant.{name}.q"] = bits(it.q)
        out[f"quant.{name}.scale"] = bits(it.scale)
    # int32 accumulators (torch._int_mm on CPU, the arithmetic oracle of the A8W8 GEMM) and the reference's own
    # Int8Linear.forward (dequantise + F.linear) output for the same activations, a loose cross-check
    xq = Int8Tensor.quantize(gc.x)
    out["gemm.acc"] = torch._int_mm(xq.q, il.qweight.t().contiguous()).numpy()
    out["gemm.int8linear_y"] = bits(il(gc.x))

    # ---- A6: KV quantisation of an fp16 state (per state, head, token over D) and materialize()
    ac = syn.attn_case(S=2, T=160, rows=2, t=16, Hq=8, Hkv=2, D=128, seed=2)
    out["attn.digest"] = digest(ac.q, ac.k, ac.v, ac.K16, ac.V16)
    kt = Int8Tensor.quantize(ac.K16)
    vt = Int8Tensor.quantize(ac.V16)
    out["kv.kq"] = bits(kt.q)
    out["kv.ks"] = bits(kt.scale)
    out["kv.vq"] = bits(vt.q)
    out["kv.vs"] = bits(vt.scale)
    # ---- A9: Hydragen split attention (CPU branch) per state, prefix = materialize(int8).to(bf16)
    Kp = materialize(kt).to(torch.bfloat16)
    Vp = materialize(vt).to(torch.bfloat16)
    pm = torch.ones(ac.K16.shape[2], dtype=torch.bool)
    pm[:7] = False                                         # a left pad run
    pm[120:123] = False                                    # and a hole
    res = []
    for s in range(2):
        r = (ac.row_state == s).nonzero().squeeze(1)
        q = ac.q[r].transpose(1, 2)                          # (n, Hq, t, D)
        k = ac.k[r].transpose(1, 2)
        v = ac.v[r].transpose(1, 2)
        res.append(_split_attention(q, k, v, Kp[s], Vp[s], pm if s == 1 else None, 128 ** -0.5).transpose(1, 2))
    out["attn.o"] = bits(torch.cat(res, 0))                  # (R, t, Hq, D) bf16
    out["attn.pm"] = pm.numpy()

    # ---- A4: Qwen3_5RMSNorm + residual add in bf16 (the decoder layer's pre-norm block)
    g = syn.gen(3)
    H = 256
    x = torch.randn(40, H, generator=g).to(torch.bfloat16)
    res_in = torch.randn(40, H, generator=g).to(torch.bfloat16)
    nw = (torch.randn(H, generator=g) * 0.1).to(torch.bfloat16)
    out["norm.digest"] = digest(x, res_in, nw)
    norm = Qwen3_5RMSNorm(H, eps=1e-6).to(torch.bfloat16)
    norm.weight.data = nw.clone()
    h = res_in + x
    out["norm.h"] = bits(h)
    out["norm.y"] = bits(norm(h))

    # ---- q/k RMSNorm + RoPE on the gated q/k/v projection output (Qwen3_5Attention.forward :647-662)
    Hq, Hkv, D = 4, 2, 64
    M = 24
    qkv = torch.randn(M, Hq * 2 * D + 2 * Hkv * D, generator=g).to(torch.bfloat16)
    qw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16)
    kw = (torch.randn(D, generator=g) * 0.1).to(torch.bfloat16)
    pos = torch.randint(0, 300, (M,), generator=g)
    out["rope.digest"] = digest(qkv, qw, kw, pos)
    qn = Qwen3_5RMSNorm(D, eps=1e-6).to(torch.bfloat16)
    qn.weight.data = qw.clone()
    kn = Qwen3_5RMSNorm(D, eps=1e-6).to(torch.bfloat16)
    kn.weight.data = kw.clone()
    qg = qkv[:, : Hq * 2 * D].view(M, Hq, 2 * D)
    q, gate = qg[..., :D], qg[..., D:]
    q = qn(q).transpose(0, 1)                                # (Hq, M, D) as (heads, tokens)
    k = kn(qkv[:, Hq * 2 * D: Hq * 2 * D + Hkv * D].view(M, Hkv, D)).transpose(0, 1)
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextRotaryEmbedding
    rcfg = Qwen3_5TextConfig(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                             rope_parameters={"rope_type": "default", "rope_theta": 1e6, "partial_rotary_factor": 1.0})
    cos_t, sin_t = Qwen3_5TextRotaryEmbedding(rcfg)(torch.zeros(1, dtype=torch.bfloat16), pos[None])
    out["rope.cos"] = bits(cos_t[0])                          # (M, D) bf16 at each token's position
    out["rope.sin"] = bits(sin_t[0])
    q2, k2 = apply_rotary_pos_emb(q[None], k[None], cos_t, sin_t)
    out["rope.q"] = bits(q2[0].transpose(0, 1))              # (M, Hq, D)
    out["rope.k"] = bits(k2[0].transpose(0, 1))
    o = torch.randn(M, Hq * D, generator=g).to(torch.bfloat16)
    out["gate.digest"] = digest(o)
    out["gate.g"] = bits(o * torch.sigmoid(gate.reshape(M, Hq * D)))

    # ---- int8 embedding table (Int8Embedding.forward, quant.py:199-200)
    emb = nn.Embedding(100, 64)
    emb.weight.data = (torch.randn(100, 64, generator=g) * 0.02).to(torch.bfloat16)
    ie = Int8Embedding(emb)
    ids = torch.randint(0, 100, (33,), generator=g)
    out["embed.digest"] = digest(emb.weight.data, ids)
    out["embed.qweight"] = bits(ie.qweight)
    out["embed.scale"] = bits(ie.scale)
    out["embed.out"] = bits(ie(ids))

    # ---- A13: Decider._probs readout + _normalize with the explicit `none` column
    N, Kmax = 6, 9
    nopt = [3, 9, 2, 5, 8, 4]
    types = ["choice", "choice", "noul", "score", "choice", "score"]
    logits = torch.randn(N, Kmax, generator=g) * 3
    mask = torch.arange(Kmax)[None, :] < torch.tensor(nopt)[:, None]
    logits = logits.masked_fill(~mask, -1e9)
    stub = nn.Module()
    stub.cfg = SimpleNamespace(noul_mode="choice")
    stub.run = lambda qs, mem: (None, DecisionOutput(logits, mask))
    qs = []
    for i in range(N):
        qq = Question(f"q{i}", [f"o{j}" for j in range(nopt[i])], types[i])
        if i % 2 == 0:
            qq.none_col = nopt[i] - 1                         # the `none` text option is the last one
        qs.append(qq)
    temps = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}
    dec = Decider(stub, temperature=1.419344425201416, temperature_by_type=temps)
    mean, _ = dec._probs(qs, None, SamplerConfig())
    out["readout.logits"] = logits.numpy()
    out["readout.mask"] = mask.numpy()
    out["readout.T"] = np.array([temps[t] for t in types], dtype=np.float32)
    out["readout.none_col"] = np.array([getattr(q, "none_col", -1) for q in qs], dtype=np.int32)
    out["readout.p"] = mean.numpy()
    ren = np.zeros((N, Kmax), dtype=np.float64)
    for i, q in enumerate(qs):
        K = getattr(q, "none_col", len(q.options))
        ren[i, :K] = _normalize(mean[i, :K])
    out["readout.renorm"] = ren

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ops.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
