"""Requests data-parallel over the GPUs of one box: one process per GPU (torchrun), replicated weights, no
data-path collective; the per-question probabilities are gathered once per batch over NCCL (gloo on CPU in tests).

shard(): contiguous blocks balanced by token count (state + question tokens), so gathering in rank order restores the
request order. gather_rows(): variable-size (n_i, K_i) blocks from every rank, padded to the largest, one all_gather,
unpadded on arrival.
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


def request_weight(req, tok) -> int:
    """Tokens a request costs: its state plus every question's prompt and options (the row passes)."""
    n = len(tok([req.state], add_special_tokens=False)["input_ids"][0])
    for q in req.questions:
        n += len(tok([q.prompt] + list(q.options), add_special_tokens=False)["input_ids"][0])
    return n


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
    renormalisation and P(none), so every rank answers exactly as one rank deciding the whole list would."""

    def __init__(self, decider, group=None):
        self.decider, self.group = decider, group

    def decide_many(self, requests) -> list:
        world, rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        tok = self.decider.model.tok
        blocks = shard([request_weight(r, tok) for r in requests], world)
        a, b = blocks[rank]
        mine = requests[a:b]
        if mine and any(r.questions for r in mine):
            plan = self.decider.plan(mine)
            (probs, renorm, p_none), _ = self.decider.execute(plan)
            # [raw probs (K) | renormalised (K) | P(none)] in float64: fp32 values and the fp64 renormalisation
            # travel exactly
            local = torch.cat([probs.double(), renorm.double(), p_none.double()[:, None]], 1)
        else:
            local = torch.zeros(0, 1, dtype=torch.float64, device=self.decider.model.backbone.device)
        parts = gather_rows(local, self.group)
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
