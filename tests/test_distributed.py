"""Host logic of the multi-GPU path with world-size-2 gloo ranks on CPU: contiguous balanced shards and the
variable-size gather that restores request order."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from opendecider_b200.distributed import gather_rows, shard


def test_shard_contiguous_balanced():
    w = [5, 1, 1, 1, 1, 1, 5, 5]
    b = shard(w, 2)
    assert b[0][0] == 0 and b[-1][1] == len(w) and b[0][1] == b[1][0]
    tot = [sum(w[s:e]) for s, e in b]
    assert abs(tot[0] - tot[1]) <= max(w)
    assert shard([1] * 8, 4) == [(0, 2), (2, 4), (4, 6), (6, 8)]
    b = shard([1, 1], 4)                       # more ranks than items: empty blocks at the end
    assert sum(e - s for s, e in b) == 2 and len(b) == 4


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = torch.full((rank + 2, 3 + rank), float(rank), dtype=torch.float64)
        parts = gather_rows(x)
        ok = [p.shape == (r + 2, 3 + r) and bool((p == r).all()) for r, p in enumerate(parts)]
        q.put((rank, all(ok)))
    finally:
        dist.destroy_process_group()


def test_gather_rows_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}


def _failing_worker(rank, world, port, q):
    """Rank 1 dies before the gather; rank 0's gather must end with an error (a short process-group timeout or the
    closed connection), never wait for good."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        q.put((rank, "died"))
        q.close()
        q.join_thread()                                      # the message is out before the process ends
        os._exit(3)                                          # leaves without joining the collective
    try:
        gather_rows(torch.zeros(2, 3))
        q.put((rank, "no error"))
    except Exception as e:                                   # noqa: BLE001 - any error is the expected outcome
        q.put((rank, "error: " + type(e).__name__))


def test_gather_fails_cleanly_when_a_rank_dies():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 500) % 1000
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "died"
    assert res[0].startswith("error"), res[0]


class _StubModel:
    """Stands in for V3Model on CPU: a tokenizer and a device; the stub decider computes its probabilities itself."""

    def __init__(self):
        from opendecider_b200.synthetic import SyntheticTokenizer
        self.tok = SyntheticTokenizer(1024)
        self.backbone = type("BB", (), {"device": torch.device("cpu")})()


def _stub_decider():
    """Decider whose device work is replaced by a deterministic CPU function of each question (the host logic -
    plans, `none`, answers - is the real Decider's). The question 'tie' gets raw probabilities [0.3, 0.3 | none 0.4]:
    P(none) beats the raw option maximum (0.3) but not the renormalised one (0.5)."""
    from opendecider_b200.decider import Decider

    class StubDecider(Decider):
        def __init__(self):
            self.model, self.temperature, self.temperature_by_type = _StubModel(), 1.0, {}
            self.none_text = "none of the above"

        def plan(self, requests, cache=None, appends=None):
            return self.plan_questions(requests)

        def execute(self, plan, cache=None):
            qs = plan["questions"]
            Kmax = max(len(q.options) for q in qs)
            probs = torch.zeros(len(qs), Kmax, dtype=torch.float32)
            for i, q in enumerate(qs):
                K = len(q.options)
                if q.prompt == "tie":
                    probs[i, :K] = torch.tensor([0.3, 0.3, 0.4])
                else:
                    w = torch.tensor([1.0 + (sum(map(ord, q.prompt + o)) % 7) for o in q.options])
                    probs[i, :K] = w / w.sum()
            renorm = torch.zeros(len(qs), Kmax, dtype=torch.float64)
            p_none = torch.zeros(len(qs), dtype=torch.float32)
            for i, q in enumerate(qs):
                K = getattr(q, "none_col", len(q.options))
                renorm[i, :K] = probs[i, :K].double() / probs[i, :K].double().sum()
                p_none[i] = probs[i, K] if hasattr(q, "none_col") else 0.0
            return (probs, renorm, p_none), None

        def decide_stream(self, batches, gather=None, cache=None):
            # Decider.decide_stream's contract without CUDA events or pinned buffers: gather() right after a
            # batch's device work, before the next batch is planned
            for item in batches:
                plan = self.plan(item)
                probs, _ = self.execute(plan)
                g = gather(probs) if gather is not None else None
                yield self.answers(plan, probs), g

    return StubDecider()


def _requests():
    from opendecider_b200.batching import Question
    from opendecider_b200.synthetic import Request
    reqs = []
    for i in range(7):
        qs = [Question(f"t{10 + i} t{11 + i}", [f"t{20 + j}" for j in range(2 + i % 3)], name="a")]
        if i % 2:
            qs.append(Question.noul(f"t{30 + i}", name="b"))
        reqs.append(Request(" ".join(f"t{40 + j}" for j in range(3 + 5 * i)), qs))
    reqs[3] = Request("t1 t2", [Question("tie", ["t5", "t6"], name="a")])
    reqs.append(Request("t3", []))                           # a request without questions
    return reqs


def _decider_worker(rank, world, port, q):
    from opendecider_b200.distributed import DistributedDecider
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dd = DistributedDecider(_stub_decider())
        reqs = _requests()
        got = dd.decide_many(reqs)
        streamed = list(dd.decide_stream([reqs[:-1], reqs[2:6], reqs[:-1]]))
        q.put((rank, (got, streamed)))
    finally:
        dist.destroy_process_group()


def test_distributed_decider_equals_single_rank():
    """DistributedDecider.decide_many on two gloo ranks answers every request exactly as one rank's decide_many:
    same values, probabilities and P(none), in request order, on both ranks - including the question whose P(none)
    beats the raw option maximum but not the renormalised one (value 'none'). decide_stream over three batches of
    different sizes answers each as decide_many does."""
    want = _stub_decider().decide_many(_requests())
    assert want[3]["a"]["value"] == "none" and want[-1] == {}
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() + 250) % 1000
    procs = [ctx.Process(target=_decider_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    single = _stub_decider()
    want_stream = [single.decide_many(b) for b in ([*_requests()[:-1]], _requests()[2:6], [*_requests()[:-1]])]
    for r in (0, 1):
        got, streamed = res[r]
        assert got == want
        assert streamed == want_stream             # the pipelined form: every batch, in order, on every rank
