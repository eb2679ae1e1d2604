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

import re
import zlib

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


# ------------------------------------------------------------------------------------------------ decision requests
class SyntheticTokenizer:
    """Deterministic word-level tokenizer standing in for the Qwen tokenizer (absent: no network) on synthetic
    workloads. A word `t<id>` is token id (mod vocab), a newline is 1, any other word (the templates' fixed words)
    is 2 + crc32(word) % 14; ids 16.. are free for random content. Has the HF tokenizer surface the reference uses:
    __call__(texts, add_special_tokens=False)["input_ids"], pad_token_id, __len__."""

    pad_token_id = 0

    _WORDS = re.compile(r"\n|[^\s]+")

    def __init__(self, vocab: int):
        self.vocab = vocab
        self._fixed = {"\n": 1}          # template words seen so far -> id

    def __len__(self) -> int:
        return self.vocab

    def encode(self, text: str) -> list:
        out = []
        V, fixed = self.vocab, self._fixed
        for w in self._WORDS.findall(text):
            d = w[1:]
            if w[0] == "t" and d.isdecimal():                # the word t<id> (decimal digits, as t\d+ matches)
                out.append(int(d) % V)
            else:
                i = fixed.get(w)
                if i is None:
                    i = fixed[w] = 2 + zlib.crc32(w.encode()) % 14
                out.append(i)
        return out

    def __call__(self, texts, add_special_tokens: bool = False):
        if isinstance(texts, str):
            return {"input_ids": self.encode(texts)}
        return {"input_ids": [self.encode(t) for t in texts]}


def words(ids) -> str:
    return " ".join(f"t{int(i)}" for i in ids)


@dataclass
class Request:
    """One decision request: a state and its questions (the atomic part of the reference's DecideRequest); `append`:
    text appended to an already-encoded state before the questions (config 5's incremental records)."""
    state: str
    questions: list
    append: str = ""


def _ids(g, n, vocab):
    return torch.randint(16, vocab, (n,), generator=g).tolist()


def _distinct_options(g, k, n_tok, vocab):
    seen, out = set(), []
    while len(out) < k:
        o = words(_ids(g, n_tok, vocab))
        if o not in seen:
            seen.add(o)
            out.append(o)
    return out


def decision_requests(config: int, seed: int = 0, n_requests: int | None = None, vocab: int | None = None,
                      state_tokens: int | None = None, n_options: int | None = None, append_tokens: int | None = None):
    """Seeded requests of BASELINE configs 1, 4 and 5 (states of random ids; state_text() adds 3 template tokens,
    so the random part is state_tokens - 3 ids and the tokenised state is exactly state_tokens long).
      1: 4 requests, 256-token states, one choice question: prompt 16 ids, 8 options x 8 ids
      4: 64 requests, 2048-token states, three questions: choice 16 options x 12 ids, yes/no, score 5 levels x
         2 ids; prompts 16 ids
      5: 512 requests, 16384-token states (+512 appended record ids, Request.append), one choice question 255
         options x 12 ids
    Returns (requests, tokenizer)."""
    from .batching import Question
    g = gen(seed)
    if config == 1:
        n, V, T, K = n_requests or 4, vocab or 1024, state_tokens or 256, n_options or 8
    elif config == 4:
        n, V, T, K = n_requests or 64, vocab or 151936, state_tokens or 2048, n_options or 16
    elif config == 5:
        n, V, T, K = n_requests or 512, vocab or 151936, state_tokens or 16384, n_options or 255
        A = 512 if append_tokens is None else append_tokens
    else:
        raise ValueError(config)
    tok = SyntheticTokenizer(V)
    reqs = []
    for i in range(n):
        state = words(_ids(g, T - 3, V))
        qs = []
        if config == 1:
            qs.append(Question(words(_ids(g, 16, V)), _distinct_options(g, K, 8, V), "choice", name="q0"))
        elif config == 4:
            qs.append(Question(words(_ids(g, 16, V)), _distinct_options(g, K, 12, V), "choice", name="choice"))
            qs.append(Question.noul(words(_ids(g, 16, V)), name="yesno"))
            qs.append(Question.score(words(_ids(g, 16, V)), _distinct_options(g, 5, 2, V), name="score"))
        else:
            qs.append(Question(words(_ids(g, 16, V)), _distinct_options(g, K, 12, V), "choice", name="choice"))
        reqs.append(Request(state, qs, words(_ids(g, A, V)) if config == 5 else ""))
    return reqs, tok
