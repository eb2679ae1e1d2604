"""Seeded synthetic workloads of the benchmark configurations (no dataset is involved; all inputs are random).

Every generator draws on the CPU from torch.Generator().manual_seed(seed), so the CUDA path, the CPU oracle and the
golden-fixture generator see identical bytes for the same arguments.

Operator configurations (shapes of the reference's hot path):
  gemm_case   W8A8 projection GEMM: X ~ N(0, 1) (M, K) with 1% of its channels scaled x20 (outliers), cast to bf16;
              W ~ N(0, 0.02) (N, K) cast to bf16, quantised per output channel (Int8Linear's layout).
  attn_case   branched shared-prefix attention: state K, V ~ N(0, 1) fp32 -> fp16 -> int8 per (state, head, token)
              with fp16 scales; option-row q and own k, v ~ N(0, 1) in bf16.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def quantize_rows_cpu(x: torch.Tensor):
    """The reference quantiser's formula on CPU tensors, for building weights at load time in generators.
    (Int8Tensor.quantize / Int8Linear.__init__, quant.py:37-41 / 124-127.) Returns (q int8, fp32 scale)."""
    xf = x.float()
    s = xf.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 127.0
    q = torch.round(xf / s).clamp_(-127, 127).to(torch.int8)
    return q, s


@dataclass
class GemmCase:
    x: torch.Tensor          # (M, K) bf16 activations
    w: torch.Tensor          # (N, K) bf16 weight
    qweight: torch.Tensor    # (N, K) int8
    wscale: torch.Tensor     # (N, 1) bf16


def gemm_case(M: int, N: int, K: int, seed: int = 0) -> GemmCase:
    g = gen(seed)
    x = torch.randn(M, K, generator=g)
    outl = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, outl] *= 20.0
    x = x.to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    q, s = quantize_rows_cpu(w)
    return GemmCase(x, w, q, s.to(torch.bfloat16))


@dataclass
class AttnCase:
    q: torch.Tensor          # (R, t, Hq, D) bf16, R = S * rows
    k: torch.Tensor          # (R, t, Hkv, D) bf16 own keys
    v: torch.Tensor          # (R, t, Hkv, D) bf16
    K16: torch.Tensor        # (S, Hkv, T, D) fp16 state keys before quantisation
    V16: torch.Tensor
    Kq: torch.Tensor         # (S, Hkv, T, D) int8
    Vq: torch.Tensor
    ks: torch.Tensor         # (S, Hkv, T, 1) fp16
    vs: torch.Tensor
    row_state: torch.Tensor  # (R,) int32


def attn_case(S: int, T: int, rows: int, t: int, Hq: int, Hkv: int, D: int, seed: int = 0) -> AttnCase:
    g = gen(seed)
    K16 = torch.randn(S, Hkv, T, D, generator=g).to(torch.float16)
    V16 = torch.randn(S, Hkv, T, D, generator=g).to(torch.float16)
    Kq, ks = quantize_rows_cpu(K16)
    Vq, vs = quantize_rows_cpu(V16)
    R = S * rows
    q = torch.randn(R, t, Hq, D, generator=g).to(torch.bfloat16)
    k = torch.randn(R, t, Hkv, D, generator=g).to(torch.bfloat16)
    v = torch.randn(R, t, Hkv, D, generator=g).to(torch.bfloat16)
    row_state = torch.arange(S, dtype=torch.int32).repeat_interleave(rows)
    return AttnCase(q, k, v, K16, V16, Kq, Vq, ks.to(torch.float16), vs.to(torch.float16), row_state)
