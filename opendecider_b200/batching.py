"""Questions, the text templates the backbone reads, and the vectorised segment layout of the row passes.

These have to stay identical to the reference for the same token ids to reach the kernels:
  Question                  src/opendecider/batching.py:16-33 (prompt, options, type, label, state_idx, name)
  state/answer templates    src/opendecider/formatting.py:10-14, 32-45 (answer row format, canonical listing)
  segment_layout            src/opendecider/cache.py:14-28 (token destinations from CPU lengths, no GPU sync)
  MAX_OPTIONS               src/opendecider/options.py:11-12 (255: the `none` option is not added at the cap)
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Any, Sequence

import torch

YES_NO = ("yes", "no")
MAX_OPTIONS = 255


@dataclass
class Question:
    prompt: str
    options: list
    type: str = "choice"            # choice | noul | score
    label: int | None = None
    state_idx: int = 0              # which state (request) of the batch this question reads
    name: str = ""

    @classmethod
    def noul(cls, prompt: str, **kw) -> "Question":
        return cls(prompt, list(YES_NO), "noul", **kw)

    @classmethod
    def score(cls, prompt: str, levels: Sequence[str], **kw) -> "Question":
        return cls(prompt, list(levels), "score", **kw)


def state_text(state: Any) -> str:
    if isinstance(state, str):
        return "State:\n" + state.strip() + "\n"
    return "State:\n" + json.dumps(state, ensure_ascii=False, separators=(",", ": ")) + "\n"


def answer_option_text(option: str) -> str:
    """An option as it follows "Answer:" (leading space)."""
    return " " + option.strip()


def answer_row_prefix(prompt: str, options, list_cap: int = 16) -> str:
    """The answer-format question row: the prompt, the candidates listed once each in case-insensitive sorted order
    (never the caller's order) when there are at most list_cap of them, then the answer cue."""
    head = "\nQuestion: " + prompt.strip()
    if 0 < len(options) <= list_cap:
        uniq = sorted({o.strip() for o in options}, key=lambda x: (x.lower(), x))
        head += "\nOptions:" + "".join("\n- " + o for o in uniq)
    return head + "\nAnswer:"


def segment_layout(lens: torch.Tensor, group: torch.Tensor, n_groups: int):
    """Lay out variable-length segments grouped consecutively into rows. lens (M,) CPU long tokens per segment,
    group (M,) CPU long row of each segment (non-decreasing). Returns per token (row, col, seg, pos) and
    row_len (n_groups,)."""
    M = lens.numel()
    seg = torch.repeat_interleave(torch.arange(M), lens)
    start = torch.cumsum(lens, 0) - lens
    pos = torch.arange(int(lens.sum())) - start[seg]
    row_len = torch.zeros(n_groups, dtype=torch.long).index_add_(0, group, lens)
    row_start = torch.cumsum(row_len, 0) - row_len
    col = start[seg] - row_start[group[seg]] + pos
    return group[seg], col, seg, pos, row_len
