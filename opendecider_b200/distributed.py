"""Requests data-parallel over the GPUs of one box: one process per GPU (torchrun), replicated weights, no
data-path collective; the per-question probabilities are gathered once per batch over NCCL (gloo on CPU in tests).

shard(): contiguous blocks balanced by request size (request_weight: words of the state, records, prompts and
options), so gathering in rank order restores the request order. gather_blocks(): every rank's (n_i, W_i) block when
all ranks know every block's shape on the host (they all hold the full request list): padded to the largest, ONE
all_gather_into_tensor, no host synchronisation.
gather_rows(): the same when the shapes are only known locally (one extra all_gather of the shapes).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard(weights, world: int) -> list[tuple[int, int]]:
    """Split items with the given weights into `world` contiguous [start, end) blocks of near-equal total weight."""
    n = len(weights)
    total = float(sum(weights))
    bounds, acc, r = [0], 0.0, 1
    for i, w in enumerate(weights):
        acc += w
        while r < world and acc >= total * r / world and len(bounds) < world:
            bounds.append(i + 1)
            r += 1
    while len(bounds) < world:
        bounds.append(n)
    bounds.append(n)
    return [(bounds[i], bounds[i + 1]) for i in range(world)]


def _words(text: str) -> int:
    return text.count(" ") + 1 if text else 0


def request_weight(req) -> int:
    """What a request costs, for balancing: the words of its state, appended records, prompts and options - a proxy
    for their tokens that needs no tokenizer pass over every request of the global batch on every rank (a word-level
    tokenizer gives exactly one token per word; characters would weight a long token id or a long word more than the
    work it causes)."""
    from .batching import state_text
    n = _words(state_text(req.state)) + _words(getattr(req, "append", "") or "")
    for q in req.questions:
        n += _words(q.prompt) + sum(_words(o) for o in q.options)
    return n


def gather_padded(x: torch.Tensor, shapes: list, group=None) -> torch.Tensor:
    """All-gather 2-D blocks whose shapes every rank knows already (shapes[r] = (rows, width) of rank r's block; x is
    this rank's): each padded to the largest, ONE all_gather_into_tensor enqueued on the current stream without a host
    synchronisation. Returns the (world x rows_max, width_max) buffer; split_blocks() cuts it into the blocks."""
    world = dist.get_world_size(group)
    R = max(1, max(h for h, _ in shapes))
    W = max(1, max(w for _, w in shapes))
    pad = torch.zeros(R, W, dtype=x.dtype, device=x.device)
    pad[: x.shape[0], : x.shape[1]] = x
    out = torch.empty(world * R, W, dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    return out


def split_blocks(buf: torch.Tensor, shapes: list) -> list[torch.Tensor]:
    """The per-rank blocks of a gather_padded buffer, in rank order."""
    R = buf.shape[0] // max(1, len(shapes))
    return [buf[r * R: r * R + h, :w] for r, (h, w) in enumerate(shapes)]


def gather_blocks(x: torch.Tensor, shapes: list, group=None) -> list[torch.Tensor]:
    """gather_padded + split_blocks: one tensor per rank, in rank order."""
    return split_blocks(gather_padded(x, shapes, group), shapes)


def gather_rows(x: torch.Tensor, group=None) -> list[torch.Tensor]:
    """All-gather a 2-D tensor whose row count and width differ across ranks. Returns one tensor per rank, in rank
    order, on every rank (padding removed)."""
    world = dist.get_world_size(group)
    dev = x.device
    shp = torch.tensor([x.shape[0], x.shape[1]], dtype=torch.int64, device=dev)
    shapes = [torch.zeros_like(shp) for _ in range(world)]
    dist.all_gather(shapes, shp, group=group)
    R = int(max(s[0] for s in shapes))
    K = int(max(s[1] for s in shapes))
    pad = torch.zeros(R, K, dtype=x.dtype, device=dev)
    pad[: x.shape[0], : x.shape[1]] = x
    outs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(outs, pad, group=group)
    return [o[: int(s[0]), : int(s[1])] for o, s in zip(outs, shapes)]


class DistributedDecider:
    """decide_many over all ranks: every rank receives the full request list, runs its contiguous block and gets
    every request's answers back. One gather per call carries, per question, the raw option probabilities (the
    softmax over the options and `none`, against which P(none) decides the value, decider.py:345), the caller-option
    renormalisation and P(none), so every rank answers exactly as one rank deciding the whole list would. Every rank
    derives every block's shape on the host (the question counts and option counts of the full list), so the gather
    is one collective with no shape exchange and no host synchronisation."""

    def __init__(self, decider, group=None):
        self.decider, self.group = decider, group

    def blocks(self, requests) -> list[tuple[int, int]]:
        return shard([request_weight(r) for r in requests], dist.get_world_size(self.group))

    def layouts(self, requests, blocks) -> list[tuple[int, int]]:
        """(questions, 2 K + 1) of every rank's gathered block: K = the block's widest option list (with `none`)."""
        out = []
        for s, e in blocks:
            qs = self.decider.plan_questions(requests[s:e])["questions"]
            K = max((len(q.options) for q in qs), default=0)
            out.append((len(qs), 2 * K + 1 if qs else 1))
        return out

    @staticmethod
    def pack(probs, renorm, p_none) -> torch.Tensor:
        """[raw probs (K) | renormalised (K) | P(none)] in float64: the fp32 values and the fp64 renormalisation
        travel exactly."""
        return torch.cat([probs.double(), renorm.double(), p_none.double()[:, None]], 1)

    def gather(self, local: torch.Tensor, shapes) -> torch.Tensor:
        """The padded all-gather of every rank's packed block (gather_padded): one collective, no host sync."""
        return gather_padded(local, shapes, self.group)

    def answers(self, requests, blocks, parts) -> list:
        out = []
        for (s, e), part in zip(blocks, parts):
            if e <= s:
                continue
            reqs = requests[s:e]
            if part.shape[0] == 0:                       # a block whose requests ask nothing
                out += [{} for _ in reqs]
                continue
            p = self.decider.plan_questions(reqs)
            K = (part.shape[1] - 1) // 2
            out += self.decider.answers(p, (part[:, :K].float(), part[:, K:2 * K], part[:, 2 * K].float()))
        return out

    def decide_many(self, requests) -> list:
        rank = dist.get_rank(self.group)
        blocks = self.blocks(requests)
        shapes = self.layouts(requests, blocks)
        a, b = blocks[rank]
        mine = requests[a:b]
        if shapes[rank][0] > 0:
            plan = self.decider.plan(mine)
            (probs, renorm, p_none), _ = self.decider.execute(plan)
            local = self.pack(probs, renorm, p_none)
        else:
            local = torch.zeros(0, 1, dtype=torch.float64, device=self.decider.model.backbone.device)
        return self.answers(requests, blocks, split_blocks(self.gather(local, shapes), shapes))

    def decide_stream(self, batches, cache=None):
        """decide_many over a sequence of request lists, pipelined as Decider.decide_stream (batch b+1 planned and
        enqueued before batch b's results are read): yields every request's answers, on every rank, per batch. With
        `cache` (this rank's block of encoded states), every batch is a (requests, appends) pair over the same
        requests, as Decider.decide_stream(cache=) takes them. Every rank's block must ask at least one question."""
        rank = dist.get_rank(self.group)
        meta = []

        def local():
            for item in batches:
                reqs = item[0] if cache is not None else item
                blocks = self.blocks(reqs)
                shapes = self.layouts(reqs, blocks)
                meta.append((reqs, blocks, shapes))
                a, b = blocks[rank]
                yield (reqs[a:b], item[1][a:b]) if cache is not None else reqs[a:b]

        def gather(probs):                               # runs right after this batch's kernels, before the next plan
            return self.gather(self.pack(*probs), meta[-1][2])

        for _, buf in self.decider.decide_stream(local(), gather=gather, cache=cache):
            reqs, blocks, shapes = meta.pop(0)
            yield self.answers(reqs, blocks, split_blocks(buf, shapes))
