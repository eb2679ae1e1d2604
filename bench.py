"""Benchmark of the B200 decision forward pass (BASELINE config 4 by default).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 4|1|5]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \\
        bench.py --gpus N --steps K --warmup W

Workload (config 4): a 9B-class dense Qwen3.5-style decoder (36 layers, hidden 4096, 32/8 heads, head_dim 128, SwiGLU
12288, vocab 151936, random-init int8 weights, int8 KV) under the V3 trunk (d_model 512, 8 heads, 4 layers, feature
layers 8/16/24/final); per GPU 64 requests, each a 2048-token random-id state with three questions (choice 16 x 12
tokens, yes/no, score 5 x 2 tokens), each + the `none` option: 192 decisions per GPU per step. One step = the whole
decision forward of that batch (state pass, question-cache row passes, trunk, readout). Requests are independent:
N GPUs decide one global batch of 64 x N requests, each its contiguous size-balanced block (weak scaling), and gather
the probabilities over NCCL.

Printed: one JSON line on rank 0. `value` = decisions/s over all GPUs with the batch's inputs resident in HBM
(device time, CUDA events, max over ranks); `e2e` = the same metric through the public API Decider.decide_stream
(one batch per step: tokenisation, one pinned host->device copy, kernels, the device->host read of the answers, the
next batch planned while the previous one runs); `roofline` = the W8A8
GEMM (the dominant kernel) timed per launch with CUDA events inside the timed region; `cpu_baseline` = the reference's
own Decider.decide_many on the host cores (the reference package installed in baseline/_ref; the bit-exact CPU port,
oracle/model.py, for config 5 or without the install) on a bounded sample, extrapolated.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TEMPS = {"choice": 1.4978350400924683, "noul": 1.2169979810714722, "score": 1.5226973295211792}
TEMPERATURE = 1.419344425201416
METRIC = "decisions/sec"


def workload(config: int):
    """(DecoderConfig, TrunkConfig kwargs, qcache threshold, description) of a bench configuration."""
    from opendecider_b200.backbone import DecoderConfig
    if config == 4:
        cfg = DecoderConfig.nine_b(feature_layers=(8, 16, 24, "final"))
        return cfg, dict(d_model=512, n_heads=8, decision_layers=4), 12, \
            "config4: 9B-class dense decoder, 64 requests/GPU x 2048-token state, 3 questions (+none)"
    if config == 5:
        cfg = DecoderConfig.nine_b(feature_layers=(8, 16, 24, "final"))
        return cfg, dict(d_model=512, n_heads=8, decision_layers=4), 12, \
            ("config5: 9B-class dense decoder, 64 requests/GPU x 16384-token cached int8 state + 512 appended "
             "tokens, 1 choice question x 255 options (no none option at the 255-option cap)")
    cfg = DecoderConfig.tiny(feature_layers=(1, 3, "final"))
    return cfg, dict(d_model=64, n_heads=4, decision_layers=2), 32, \
        "config1: tiny decoder, 4 requests x 256-token state, 1 choice question x 8 options (+none)"


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region (rank 0, all GPUs of the run)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_gpus: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        ids = ",".join(str(i) for i in range(n_gpus))
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", ids, f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [l.strip().split(", ") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        load = [s for s in sm if mx and s > 0.3 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------------ CPU oracle
class CpuSample:
    """The CPU oracle (oracle/model.py: bit-exact with the reference's own decide_many on config 1 and the edge batch)
    timed on one request of the workload at two depths, n_lo and n_hi decoder layers (layers past the first reuse
    layer 0's weights: timing only). The slope between the two is the cost of one layer, the intercept the fixed cost
    (embedding, trunk, readout); one request = intercept + all layers x slope. The decoder's feature layers are read
    from the last sampled layer (same shapes and trunk work)."""

    def __init__(self, config: int, n_lo: int = 2, n_hi: int = 8, seed: int = 0):
        from oracle.model import OracleDecision
        from opendecider_b200 import synthetic as syn
        from opendecider_b200.backbone import synthetic_weights
        from opendecider_b200.v3 import TrunkConfig, trunk_state_dict
        from oracle.trunk import OracleTrunk
        torch.set_num_threads(os.cpu_count() or 1)
        cfg, tk, qmin, _ = workload(config)
        self.cfg, self.n_layers_total = cfg, cfg.layers
        self.n_lo, self.n_hi = min(n_lo, cfg.layers), min(n_hi, cfg.layers)
        self.reqs, tok = syn.decision_requests(config, seed=seed, n_requests=1)
        tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(cfg.feature_layers), **tk)
        trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
        sd = synthetic_weights(cfg, seed=0, layers=1)
        self.feats = cfg.feature_layers
        cfg.feature_layers = ("final",) * len(self.feats)
        self.od = OracleDecision(cfg, sd, trunk, tok, TEMPS, TEMPERATURE, layers=1, qcache_min_rows=qmin)
        for table in (self.od.dec.q, self.od.dec.norm):   # layers 1..n_hi-1 alias layer 0's quantised weights
            table.update(self._alias(table, self.n_hi))   # (runs its first n layers when od.dec.n = n)
        self._time(self.n_lo)                         # warm-up: allocator, thread pool, kernel selection

    @staticmethod
    def _alias(sd, n):
        """Layers 1..n-1 reuse layer 0's weights (timing only: the sample is not checked for parity)."""
        out = dict(sd)
        for k, v in sd.items():
            if k.startswith("layers.0"):
                for i in range(1, n):
                    out[k.replace("layers.0.", f"layers.{i}.", 1)] = v
        return out

    def _time(self, n: int) -> float:
        self.od.dec.n = n
        t0 = time.perf_counter()
        self.od.decide(self.reqs)
        return time.perf_counter() - t0

    def step(self):
        """One timed sample. Returns (decisions/s of the whole-depth request, threads, description)."""
        t_lo, t_hi = self._time(self.n_lo), self._time(self.n_hi)
        per_layer = max(0.0, (t_hi - t_lo) / max(1, self.n_hi - self.n_lo))
        fixed = max(0.0, t_lo - self.n_lo * per_layer)
        t_req = fixed + self.n_layers_total * per_layer
        nd = sum(len(r.questions) for r in self.reqs)
        desc = (f"oracle/model.py (PyTorch CPU: int8 _int_mm projections, torch's CPU attention) on 1 request "
                f"({nd} decisions) timed at {self.n_lo} and {self.n_hi} of {self.n_layers_total} decoder layers "
                f"({t_lo:.1f} s, {t_hi:.1f} s): {per_layer:.2f} s per layer + {fixed:.2f} s fixed, extrapolated to "
                f"all layers ({t_req:.1f} s per request)")
        return nd / t_req, torch.get_num_threads(), desc


class CpuSampleCached:
    """Config 5 on the CPU oracle: one request whose 16384-token state is already cached (the timed work is the
    append of 512 tokens and the decision, as in the B200 arm; the cache content does not change the cost, so it is
    random int8 rows materialised). The oracle runs option rows one at a time, so the request is timed with 2 and
    with 6 options and the row cost extrapolated linearly to the workload's 256 rows (255 options + none), and the
    layers sampled extrapolated linearly to all layers."""

    K_SMALL, K_LARGE = 2, 6

    def __init__(self, budget_s: float, seed: int = 0):
        from oracle.model import OracleDecision
        from oracle import ops
        from opendecider_b200 import synthetic as syn
        from opendecider_b200.backbone import synthetic_weights
        from opendecider_b200.v3 import TrunkConfig, trunk_state_dict
        from oracle.trunk import OracleTrunk
        torch.set_num_threads(os.cpu_count() or 1)
        cfg, tk, qmin, _ = workload(5)
        self.cfg, self.n_layers_total = cfg, cfg.layers
        full, tok = syn.decision_requests(5, seed=seed, n_requests=1)
        self.rows_full = len(full[0].questions[0].options) + 1
        self.reqs = {k: syn.decision_requests(5, seed=seed, n_requests=1, n_options=k)[0][0]
                     for k in (self.K_SMALL, self.K_LARGE)}
        self.T = len(tok([full[0].state], add_special_tokens=False)["input_ids"][0]) + 3
        tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(cfg.feature_layers), **tk)
        trunk = OracleTrunk(tc, trunk_state_dict(tc, seed=0))
        sd = synthetic_weights(cfg, seed=0, layers=1)
        self.feats = cfg.feature_layers
        cfg.feature_layers = ("final",) * len(self.feats)
        g = torch.Generator().manual_seed(seed)
        shp = (1, cfg.kv_heads, self.T, cfg.head_dim)

        def rnd():
            q = torch.randint(-127, 128, shp, generator=g, dtype=torch.int8)
            return ops.materialize_int8(q, torch.full(shp[:-1] + (1,), 0.01, dtype=torch.bfloat16))

        self.kv1 = (rnd(), rnd())
        mk = lambda n: OracleDecision(cfg, CpuSample._alias(sd, n), trunk, tok, TEMPS, TEMPERATURE, layers=n,
                                      qcache_min_rows=qmin)
        t1 = self._time(mk(1), self.K_LARGE)
        self.n = max(1, min(cfg.layers, int(budget_s / max(2.0 * t1, 1e-3))))
        self.od = mk(self.n)

    def _time(self, od, k) -> float:
        pre = ([self.kv1] * od.dec.n, torch.zeros(1, dtype=torch.long), self.T, [self.T])
        r = self.reqs[k]
        t0 = time.perf_counter()
        nxt, _, _ = od.append_pass(pre, [r.append])
        od.decide([r], prebuilt=nxt)
        return time.perf_counter() - t0

    def step(self):
        ts, tl = self._time(self.od, self.K_SMALL), self._time(self.od, self.K_LARGE)
        per_row = max(0.0, (tl - ts) / (self.K_LARGE - self.K_SMALL))
        t_req = (ts + per_row * (self.rows_full - self.K_SMALL - 1)) * self.n_layers_total / self.n
        desc = (f"oracle/model.py (PyTorch CPU) on 1 request with a cached {self.T}-token state: append + decision "
                f"timed with {self.K_SMALL} and {self.K_LARGE} options ({ts:.1f} s, {tl:.1f} s) over {self.n} of "
                f"{self.n_layers_total} layers, extrapolated linearly to {self.rows_full} option rows and all layers")
        return 1.0 / t_req, torch.get_num_threads(), desc


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def reference_installed() -> bool:
    return os.path.isdir(os.path.join(REF_DIR, "opendecider"))


class RefCpuSample:
    """The reference's OWN code timed on the host cores: `opendecider.decider.Decider.decide_many` from the unmodified
    reference package installed in baseline/_ref, on its stock CPU path (int8 weight-only linears dequantised per
    call, `Int8Linear.forward` quant.py:149-157; the state pass, question cache and option rows of decide_many,
    decider.py:438-484; torch's CPU attention). Set-up only, none of which changes the arithmetic: a Qwen3.5 text
    model built from the workload's configuration (every layer full attention, HF random init, bf16) instead of a
    checkpoint, the reference's quantize_int8_ / Int8Embedding, its use_reference_kernels(True), a no-op
    `_update_linear_attn_mask` (transformers 5.5 raises on an all-attention cache), the word-level synthetic tokenizer.
    One request of the workload is decided at n_lo and n_hi decoder layers (layers past the first share its int8
    weights: timing only); the slope is one layer's cost and the intercept the fixed cost, extrapolated to all layers.
    The trunk reads its feature layers from the last sampled layer (same shapes and work)."""

    def __init__(self, config: int, n_lo: int = 2, n_hi: int = 10, seed: int = 0):
        if not reference_installed():
            raise RuntimeError("the reference package is not installed in baseline/_ref")
        if REF_DIR not in sys.path:
            sys.path.insert(0, REF_DIR)
        from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
        from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5ForCausalLM, Qwen3_5TextModel
        from opendecider.backbone import Backbone, BackboneConfig, use_reference_kernels
        from opendecider.decider import Decider, prepare_inference_
        from opendecider.models import ModelConfig, build_model
        from opendecider.quant import Int8Embedding, quantize_int8_
        from opendecider_b200 import synthetic as syn
        from opendecider_b200.backbone import synthetic_weights
        torch.set_num_threads(os.cpu_count() or 1)
        cfg, tk, _, _ = workload(config)
        self.n_layers_total = cfg.layers
        self.n_lo, self.n_hi = min(n_lo, cfg.layers), min(n_hi, cfg.layers)
        reqs, tok = syn.decision_requests(config, seed=seed, n_requests=1)
        self.nd = sum(len(r.questions) for r in reqs)
        self.reqs = [{"state": r.state, "questions": {q.name: self._question(q) for q in r.questions}} for r in reqs]
        use_reference_kernels(True)
        Qwen3_5TextModel._update_linear_attn_mask = lambda self, am, pkv: None
        c = Qwen3_5TextConfig(
            vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=1,
            num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
            layer_types=["full_attention"], rms_norm_eps=cfg.eps, tie_word_embeddings=True,
            pad_token_id=tok.pad_token_id,
            rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta, "partial_rotary_factor": 1.0})
        # built on the meta device and filled with the seeded synthetic weights (HF's own random init of the 0.6 G
        # embedding takes a minute on the CPU); the rotary table is built on the CPU in fp32, as from_pretrained keeps it
        dt = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device("meta"):
                lm = Qwen3_5ForCausalLM(c).model
        finally:
            torch.set_default_dtype(dt)
        lm = lm.to_empty(device="cpu").eval()
        lm.rotary_emb = type(lm.rotary_emb)(config=c)
        missing, unexpected = lm.load_state_dict(synthetic_weights(cfg, seed=seed, layers=1), strict=False)
        assert not unexpected and not missing, (missing, unexpected)
        quantize_int8_(lm.layers)
        lm.embed_tokens = Int8Embedding(lm.embed_tokens)
        self.lm, self.layer0 = lm, lm.layers[0]
        self.share = {id(t): t for t in list(self.layer0.parameters()) + list(self.layer0.buffers())}
        self.tok, self.Backbone, self.BackboneConfig = tok, Backbone, BackboneConfig
        self.mcfg = lambda: ModelConfig(variant="v3", slot_emb="none", dropout=0.0, v3_features="branched",
                                        v3_row_format="answer", v3_cross="question", v3_layer_combine="mix",
                                        v3_lm_feature=False, **tk)
        self.build_model, self.prepare_inference_, self.Decider = build_model, prepare_inference_, Decider
        self.n_feat = len(cfg.feature_layers)
        self.deciders = {n: self._decider(n) for n in (self.n_lo, self.n_hi)}
        self._time(self.n_lo)                          # warm-up: allocator, thread pool, kernel selection
        self._time(self.n_hi)

    @staticmethod
    def _question(q) -> dict:
        """A synthetic question in the reference's request schema (schema.py: choice options, noul, score levels)."""
        if q.type == "noul":
            return {"type": "noul", "prompt": q.prompt}
        if q.type == "score":
            return {"type": "score", "prompt": q.prompt, "levels": list(q.options)}
        return {"type": q.type, "prompt": q.prompt, "options": list(q.options)}

    def _decider(self, n: int):
        import copy
        layers = [self.layer0]
        for i in range(1, n):
            lay = copy.deepcopy(self.layer0, dict(self.share))
            lay.self_attn.layer_idx = i
            layers.append(lay)
        self.lm.layers = torch.nn.ModuleList(layers)
        self.lm.config.num_hidden_layers = n
        self.lm.config.layer_types = ["full_attention"] * n
        bcfg = self.BackboneConfig(path="synthetic", dtype="bfloat16", weight_quant="int8", kv_quant="int8",
                                   feature_layers=["final"] * self.n_feat, device="cpu")
        lm = copy.copy(self.lm)                        # its own layer list and config; shared weights
        lm._modules = dict(self.lm._modules)
        lm.config = copy.copy(self.lm.config)
        bb = self.Backbone(lm, self.tok, bcfg)
        torch.manual_seed(0)
        model = self.build_model(bb, self.mcfg()).eval()
        self.prepare_inference_(model)
        return self.Decider(model, temperature=TEMPERATURE, temperature_by_type=TEMPS)

    def _time(self, n: int) -> float:
        t0 = time.perf_counter()
        with torch.inference_mode():
            ans = self.deciders[n].decide_many(self.reqs)
        dt = time.perf_counter() - t0
        assert len(ans) == len(self.reqs)
        return dt

    def step(self, reps: int = 3):
        """One timed sample: the median of `reps` timings at each depth. Returns (decisions/s of the whole-depth
        request, threads, description)."""
        t_lo = statistics.median(self._time(self.n_lo) for _ in range(reps))
        t_hi = statistics.median(self._time(self.n_hi) for _ in range(reps))
        per_layer = max(0.0, (t_hi - t_lo) / max(1, self.n_hi - self.n_lo))
        fixed = max(0.0, t_lo - self.n_lo * per_layer)
        t_req = fixed + self.n_layers_total * per_layer
        desc = (f"the reference's own Decider.decide_many (baseline/_ref, stock CPU path: int8 weight-only linears, "
                f"torch CPU attention) on 1 request ({self.nd} decisions) timed at {self.n_lo} and {self.n_hi} of "
                f"{self.n_layers_total} decoder layers (medians of 3: {t_lo:.2f} s, {t_hi:.2f} s): {per_layer:.3f} s per "
                f"layer + {fixed:.2f} s fixed, extrapolated to all layers ({t_req:.1f} s per request)")
        return self.nd / t_req, torch.get_num_threads(), desc


def cpu_oracle_sample(config: int, budget_s: float):
    if config == 5:
        return CpuSampleCached(budget_s).step()
    return CpuSample(config).step()


def cpu_baseline_sample(config: int, budget_s: float, samples: int = 3):
    """(value, threads, description, kind): the reference's own code where it is installed and the configuration is
    a plain decide_many (configs 1 and 4; the mean of `samples` timed samples), else the bit-exact port (config 5's
    cached-state append)."""
    if config != 5 and reference_installed():
        rs = RefCpuSample(config)
        got = [rs.step() for _ in range(samples)]
        return statistics.mean(g[0] for g in got), got[0][1], got[-1][2] + f"; mean of {samples} samples", "reference"
    return (*cpu_oracle_sample(config, budget_s), "port")


def run_reference(args, rank: int) -> None:
    """--impl reference: the reference's own CPU implementation of the path on the host cores - its Decider.decide_many
    from the installed reference package (RefCpuSample) for configs 1 and 4, with the bit-exact port timed once beside
    it as a cross-check; config 5 (the cached-state append) and a missing install time the port."""
    if rank != 0:
        return
    cfg, _, _, desc = workload(args.config)
    use_ref = args.config != 5 and reference_installed()
    if use_ref:
        cs, kind = RefCpuSample(args.config), "reference"
    else:
        per_step = max(3.0, 120.0 / max(1, args.steps + args.warmup))
        cs, kind = (CpuSampleCached(per_step) if args.config == 5 else CpuSample(args.config)), "port"
    vals = []
    for i in range(args.warmup + args.steps):
        v, cores, sample = cs.step()
        if i >= args.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    line = {
        "metric": METRIC, "value": value, "unit": "decisions/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
        "config": {"workload": desc, "global_batch": None},
        "cpu_baseline": {"value": value, "unit": "decisions/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "decisions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if use_ref:
        pv, pc, ps = CpuSample(args.config).step()
        line["port_cross_check"] = {"value": pv, "unit": "decisions/s", "cores": pc, "kind": "port", "sample": ps}
    print(json.dumps(line))


# ------------------------------------------------------------------------------------------------ B200 arm
def traffic_ratio():
    """DRAM bytes per algorithmic byte of the W8A8 GEMM, from the committed ncu summary of one launch
    (profiles/gemm_w8a8_pair_8192x10240x4096.md), else None."""
    path = os.path.join(ROOT, "profiles", "gemm_w8a8_pair_8192x10240x4096.md")
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("dram_bytes_per_algorithmic_byte:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def _peaks():
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(pk)) if os.path.exists(pk) else {}


def int8_peak(dev, seconds: float = 2.0) -> dict:
    """The dense int8 tensor rate measured here: cuBLASLt's int8 GEMM (torch._int_mm) at 8192^3, best of 5 single
    launches (burst) and back to back for `seconds` (sustained, as a GEMM inside a long step runs), TOP/s."""
    a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
    ops = 2.0 * 8192 ** 3
    for _ in range(3):
        torch._int_mm(a, b)
    burst = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        burst.append(ops / (e0.elapsed_time(e1) / 1e3) / 1e12)
    n = max(1, int(seconds * min(burst) * 1e12 / ops))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        torch._int_mm(a, b)
    e1.record()
    torch.cuda.synchronize()
    return {"burst": max(burst), "sustained": n * ops / (e0.elapsed_time(e1) / 1e3) / 1e12,
            "how": f"torch._int_mm (cuBLASLt int8) 8192^3: best of 5 launches, and {n} back to back"}


def _flush_l2(buf):
    """Write 256 MB (more than the 126 MB L2), then read the first half back: the write alone would leave L2 full of
    dirty lines whose write-back to HBM lands inside the next (timed) kernel; after the read L2 holds clean lines of
    the flush buffer only, none of the timed kernel's operands."""
    buf.add_(1)
    torch.sum(buf[: buf.numel() // 2], dim=0, out=buf[-1:].view(()))


def op_gemm(args):
    """the W8A8 GEMM at M in {512, 2048, 8192} x (K, N) in {(4096, 4096), (4096, 12288),
    (12288, 4096)}; one JSON line per shape (TOP/s vs 2 x measured bf16, GB/s of the algorithmic bytes,
    cuBLASLt's int8 GEMM (torch._int_mm) on the same operands for context). L2 flushed between iterations (_flush_l2)."""
    from opendecider_b200 import _lib
    from opendecider_b200 import synthetic as syn
    dev = torch.device("cuda", 0)
    shapes = [tuple(int(v) for v in x.split("x")) for x in args.shapes.split(",")] if args.shapes else \
        [(m, n, k) for m in (512, 2048, 8192) for (k, n) in ((4096, 4096), (4096, 12288), (12288, 4096))]
    peak = 2.0 * _peaks().get("bf16_tflops", 1590.0)            # burst: a kernel timed alone
    i8 = int8_peak(dev)
    print(json.dumps({"op": "int8_peak", **i8}))
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=dev)
    split_list = [int(v) for v in args.splits.split(",")] if args.splits else [None]
    for (M, N, K), sp in ((shape, sp) for shape in shapes for sp in split_list):
        gc = syn.gemm_case(M, N, K, seed=0)
        xq, sx = _lib.quant_rows(gc.x.to(dev), scale_dtype=torch.float32)
        wq, sw = gc.qweight.to(dev), gc.wscale.to(dev).view(-1)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        ts, tc = [], []
        for i in range(args.warmup + args.steps):
            _flush_l2(flush)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            _lib.gemm_w8a8(xq, sx.view(-1), wq, sw, _lib.OD_EPI_BF16, out=y, splits=sp)
            b.record()
            _flush_l2(flush)
            c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c.record()
            torch._int_mm(xq, wq.t())
            d.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
                tc.append(c.elapsed_time(d))
        assert _lib.device_error(dev) == 0, "a kernel reported a device-side error (a bounded wait ran out)"
        t = statistics.median(ts) / 1e3
        ops = 2.0 * M * N * K
        byts = M * K + N * K + 2 * M * N + 4 * M + 2 * N
        print(json.dumps({"op": "gemm_w8a8", "shape": {"M": M, "N": N, "K": K}, "ms": t * 1e3,
                          "splits": sp or _lib._gemm_plan(M, N, K, dev),
                          "tops": ops / t / 1e12, "peak_tops": peak, "frac": ops / t / 1e12 / peak,
                          "frac_of_int8_burst": ops / t / 1e12 / i8["burst"],
                          "gbs": byts / t / 1e9, "cublaslt_int8_tops": ops / (statistics.median(tc) / 1e3) / 1e12,
                          "l2": "flushed between iterations"}))


def op_attn(args):
    """branched shared-prefix attention, 32 requests x 4096-token int8 state (fp16 scales),
    32 q / 8 kv heads, D 128, 64 option rows x 16 tokens per request; plus the diagnostic bandwidth-bound shape
    (3 rows x 2 tokens per request). GB/s of the algorithmic bytes and TFLOP/s."""
    from opendecider_b200 import _lib
    dev = torch.device("cuda", 0)
    peaks = _peaks()
    shapes = ((args.requests or 32, 64, 16), (args.requests or 32, 3, 2))
    if args.shapes:
        shapes = tuple(tuple(int(v) for v in x.split("x")) for x in args.shapes.split(","))
    for S, rows, t in shapes:
        T, Hq, Hkv, D = 4096, 32, 8, 128
        g = torch.Generator(device=dev).manual_seed(0)
        K16 = torch.randn(S, Hkv, T, D, generator=g, device=dev).to(torch.float16)
        V16 = torch.randn(S, Hkv, T, D, generator=g, device=dev).to(torch.float16)
        Kq, ks = _lib.quant_rows(K16.view(-1, D))
        Vq, vs = _lib.quant_rows(V16.view(-1, D))
        del K16, V16
        R = S * rows
        q = torch.randn(R, t, Hq, D, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(R, t, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(R, t, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
        row_state = torch.arange(S, dtype=torch.int32, device=dev).repeat_interleave(rows)
        kw = dict(Kp=Kq.view(S, Hkv, T, D), Vp=Vq.view(S, Hkv, T, D), ksc=ks.view(S, Hkv, T),
                  vsc=vs.view(S, Hkv, T), row_state=row_state)
        per = max(1, min(rows, _lib.ATTN_CTA_SLOTS // (t * (Hq // Hkv))))   # rows of a request share a CTA
        starts = [(s * rows + a, min(per, rows - a)) for s in range(S) for a in range(0, rows, per)]
        kw["row_groups"] = torch.tensor(starts, dtype=torch.int32, device=dev)
        kw["max_group_rows"] = per
        out = torch.empty_like(q)
        ts = []
        for i in range(args.warmup + args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            _lib.prefix_attn(q, k, v, D ** -0.5, out=out, **kw)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        tm = statistics.median(ts) / 1e3
        flops = R * t * Hq * (T + (t + 1) / 2) * D * 4.0
        byts = S * Hkv * T * (2 * D + 2 * 2) + 2 * R * t * Hq * D * 2 + 2 * R * t * Hkv * D * 2
        print(json.dumps({"op": "prefix_attn", "shape": {"requests": S, "state_tokens": T, "rows": rows, "t": t,
                                                         "Hq": Hq, "Hkv": Hkv, "D": D},
                          "ms": tm * 1e3, "tflops": flops / tm / 1e12, "gbs": byts / tm / 1e9,
                          "frac_hbm": byts / tm / 1e9 / peaks.get("hbm_gbs", 6650.0),
                          "frac_bf16": flops / tm / 1e12 / peaks.get("bf16_tflops", 1590.0),
                          "flop_per_byte": flops / byts}))


def op_attn_state(args):
    """The state pass's attention (causal over each row's own keys, no prefix) at config-4 shapes: R rows x T tokens,
    32 q / 8 kv heads, D 128 (default 64 x 2048). TFLOP/s of the causal QK + PV FLOPs."""
    from opendecider_b200 import _lib
    dev = torch.device("cuda", 0)
    peaks = _peaks()
    shapes = [tuple(int(v) for v in x.split("x")) for x in (args.shapes or "64x2048").split(",")]
    for R, T in shapes:
        Hq, Hkv, D = 32, 8, 128
        g = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(R, T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(R, T, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
        v = torch.randn(R, T, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        ts = []
        for i in range(args.warmup + args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            _lib.prefix_attn(q, k, v, D ** -0.5, out=out)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        assert _lib.device_error(dev) == 0, "a kernel reported a device-side error"
        tm = statistics.median(ts) / 1e3
        flops = R * Hq * T * (T + 1) / 2 * D * 4.0
        byts = 2 * R * T * Hq * D * 2 + 2 * R * T * Hkv * D * 2
        print(json.dumps({"op": "prefix_attn_state", "shape": {"rows": R, "tokens": T, "Hq": Hq, "Hkv": Hkv, "D": D},
                          "ms": tm * 1e3, "tflops": flops / tm / 1e12,
                          "frac_bf16": flops / tm / 1e12 / peaks.get("bf16_tflops", 1590.0), "gbs": byts / tm / 1e9}))


def op_trunk(args):
    """The V3 trunk's kernels at the config-4 trunk shapes (d_model 512, 8 heads, xATGLU width 1368, features 4096):
    od_gemm_f32 (3xTF32: three tf32 tensor-core products per fp32 product; `tf32_frac` = 3 x 2MNK / t against half the
    measured bf16 burst rate, the tf32 dense rate of B200) beside PyTorch's fp32 GEMM on the same operands (cuBLAS,
    TF32 off), and od_trunk_attn on the option self-attention (192 questions x 200 option-token slots) beside PyTorch's
    SDPA with the materialised (N, h, P, P) float mask it replaces. L2 flushed between launches."""
    from opendecider_b200 import _lib
    dev = torch.device("cuda", 0)
    tf32_peak = 0.5 * _peaks().get("bf16_tflops", 1590.0)
    flush = torch.zeros(64 << 20, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    torch.backends.cuda.matmul.allow_tf32 = False

    def timed(fn):
        ts = []
        for i in range(args.warmup + args.steps):
            _flush_l2(flush)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        return statistics.median(ts) / 1e3

    shapes = [tuple(int(v) for v in x.split("x")) for x in args.shapes.split(",")] if args.shapes else \
        [(16384, 512, 4096), (38400, 1536, 512), (38400, 2736, 512), (38400, 512, 1368)]
    for (M, N, K) in shapes:
        x = torch.randn(M, K, generator=g, device=dev)
        w = torch.randn(N, K, generator=g, device=dev) / K ** 0.5
        b = torch.randn(N, generator=g, device=dev)
        xp, wp = _lib.split_tf32(x), _lib.split_tf32(w)
        y = torch.empty(M, N, device=dev)
        t = timed(lambda: _lib.gemm_f32(xp, wp, bias=b, out=y))
        tl = timed(lambda: torch.nn.functional.linear(x, w, b))
        fl = 2.0 * M * N * K
        print(json.dumps({"op": "gemm_f32", "shape": {"M": M, "N": N, "K": K}, "ms": t * 1e3,
                          "fp32_tflops": fl / t / 1e12, "tf32_tflops": 3 * fl / t / 1e12,
                          "tf32_frac": 3 * fl / t / 1e12 / tf32_peak, "torch_fp32_ms": tl * 1e3}))
    B, P, H, Dh = 192, 200, 8, 64
    D = H * Dh
    gid = torch.full((B, P), -1, dtype=torch.int32)
    gc = torch.Generator().manual_seed(0)
    for q in range(B):
        c = 0
        for k in range(17):
            n = int(torch.randint(1, 12, (1,), generator=gc))
            if c + n > P:
                break
            gid[q, c:c + n] = k
            c += n
    gid_d = gid.to(dev)
    qkv = torch.randn(B * P, 3 * D, generator=g, device=dev)
    bonus = torch.randn(H, generator=g, device=dev)
    olen = (gid >= 0).sum(1).int().to(dev)
    t = timed(lambda: _lib.trunk_attn(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], _lib.OD_TRUNK_SELF, B, P, P, H,
                                      k_grp=gid_d, q_grp=gid_d, bonus=bonus))
    t_len = timed(lambda: _lib.trunk_attn(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], _lib.OD_TRUNK_SELF, B, P, P,
                                          H, k_grp=gid_d, q_grp=gid_d, bonus=bonus, q_len=olen, k_len=olen))
    gl = gid_d.long()
    x_pad = gl < 0
    same = ((gl[:, :, None] == gl[:, None, :]) & ~x_pad[:, :, None]).float()
    q4 = qkv.view(B, P, 3, H, Dh)

    def sdpa():
        bias = (bonus.view(1, H, 1, 1) * same[:, None]).masked_fill(x_pad[:, None, None, :], -1e9)
        return torch.nn.functional.scaled_dot_product_attention(q4[:, :, 0].transpose(1, 2), q4[:, :, 1].transpose(1, 2),
                                                                q4[:, :, 2].transpose(1, 2), attn_mask=bias)
    ts_ = timed(sdpa)
    fl = 4.0 * B * H * P * P * Dh
    print(json.dumps({"op": "trunk_attn_self", "shape": {"questions": B, "P": P, "heads": H, "Dh": Dh},
                      "ms": t * 1e3, "tflops": fl / t / 1e12, "ms_with_row_lengths": t_len * 1e3,
                      "torch_sdpa_with_mask_ms": ts_ * 1e3}))
    assert _lib.device_error(dev) == 0, "a kernel reported a device-side error"


def op_rows(args):
    """The bandwidth-bound row kernels of a decoder layer at the 9B widths (hidden 4096, 32 / 8 heads, D 128, SwiGLU
    12288) over M tokens (default 131072, one state-pass chunk): GB/s of each kernel's algorithmic bytes (every input
    read once, every output written once; the RoPE tables and norm weights stay in L2 and are not counted) and the
    fraction of the measured HBM copy rate. Inputs are larger than L2 (126 MB), so every launch streams from HBM."""
    from opendecider_b200 import _lib
    from opendecider_b200.rope import rope_tables
    dev = torch.device("cuda", 0)
    hbm = _peaks().get("hbm_gbs", 6650.0)
    M = int(args.shapes or 131072)
    H, Hq, Hkv, D, F = 4096, 32, 8, 128, 12288
    W = Hq * D
    g = torch.Generator(device=dev).manual_seed(0)
    bf = lambda *shape: torch.randn(*shape, generator=g, device=dev).to(torch.bfloat16)
    x, res, w = bf(M, H), bf(M, H), bf(H) * 0.1
    hm = bf(M, F)
    qkv = bf(M, 2 * W + 2 * Hkv * D)
    o = bf(M, W)
    cos, sin = rope_tables(D, 1e6, 32768, torch.bfloat16, dev)
    pos = torch.randint(0, 4096, (M,), generator=g, device=dev, dtype=torch.int32)
    qn, kn = bf(D) * 0.1, bf(D) * 0.1
    S, t = M // 2048, 2048
    kq = torch.empty(S, Hkv, t, D, dtype=torch.int8, device=dev)
    vq = torch.empty_like(kq)
    ksc = torch.empty(S, Hkv, t, dtype=torch.bfloat16, device=dev)
    vsc = torch.empty_like(ksc)
    kb = torch.empty(S, Hkv, t, D, dtype=torch.bfloat16, device=dev)
    vb = torch.empty_like(kb)
    kk, vv = bf(S, t, Hkv, D), bf(S, t, Hkv, D)
    res_out = torch.empty_like(res)
    cases = [
        ("rmsnorm_res_quant", lambda: _lib.rmsnorm_res_quant(x, w, 1e-6, res_in=res, res_out=res_out),
         M * (7 * H + 4)),
        ("quant_rows", lambda: _lib.quant_rows(hm, scale_dtype=torch.float32), M * (3 * F + 4)),
        ("gate_quant", lambda: _lib.gate_quant(o, qkv, Hq, D), M * (5 * W + 4)),
        ("qk_norm_rope", lambda: _lib.qk_norm_rope(qkv, pos, cos, sin, qn, kn, 1e-6, Hq, Hkv, D),
         M * (4 * (W + 2 * Hkv * D) + 4)),
        ("kv_append", lambda: _lib.kv_append(kk, vv, kq, vq, ksc, vsc, t0=0, kb=kb, vb=vb),
         M * Hkv * (2 * D * 2 + 2 * D + 2 * 2 + 2 * D * 2)),
        ("qk_norm_rope_kv", lambda: _lib.qk_norm_rope_kv(qkv, pos, cos, sin, qn, kn, 1e-6, Hq, Hkv, D, t, kq, vq, ksc,
                                                         vsc, 0, kb=kb, vb=vb),
         M * (4 * (W + 2 * Hkv * D) + 4) + M * Hkv * (2 * D + 2 * 2 + 2 * D * 2)),
    ]
    only = set(args.kernels.split(",")) if args.kernels else None
    for name, fn, byts in cases:
        if only and name not in only:
            continue
        ts = []
        for i in range(args.warmup + args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        assert _lib.device_error(dev) == 0, "a kernel reported a device-side error"
        tm = statistics.median(ts) / 1e3
        print(json.dumps({"op": name, "tokens": M, "ms": tm * 1e3, "bytes": byts, "gbs": byts / tm / 1e9,
                          "frac_hbm": byts / tm / 1e9 / hbm}))


def op_lm_logprob(args):
    """The LM-head log-prob feature's kernel (od_lm_logprob) at the 9B head: M option tokens x V = 151936 vocabulary
    rows x H = 4096 (default M = 16384). TFLOP/s of the 2 M V H GEMM FLOPs (the log-sum-exp rides in the epilogue)."""
    from opendecider_b200 import _lib
    dev = torch.device("cuda", 0)
    peaks = _peaks()
    shapes = [tuple(int(v) for v in x.split("x")) for x in (args.shapes or "16384x151936").split(",")]
    H = 4096
    for M, V in shapes:
        g = torch.Generator(device=dev).manual_seed(0)
        h = torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16)
        qW = torch.randint(-127, 128, (V, H), generator=g, device=dev, dtype=torch.int8)
        sW = (torch.rand(V, generator=g, device=dev) * 1e-3 + 1e-4).to(torch.bfloat16)
        Wb = _lib.dequant_rows(qW, sW.view(-1, 1), torch.bfloat16)
        tok = torch.randint(0, V, (M,), generator=g, device=dev)
        ts = []
        for i in range(args.warmup + args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            _lib.lm_logprob(h, Wb, qW, sW, tok)
            b.record()
            torch.cuda.synchronize()
            if i >= args.warmup:
                ts.append(a.elapsed_time(b))
        assert _lib.device_error(dev) == 0, "a kernel reported a device-side error"
        tm = statistics.median(ts) / 1e3
        flops = 2.0 * M * V * H
        print(json.dumps({"op": "lm_logprob", "shape": {"M": M, "V": V, "H": H}, "ms": tm * 1e3,
                          "tflops": flops / tm / 1e12,
                          "frac_bf16": flops / tm / 1e12 / peaks.get("bf16_tflops", 1590.0),
                          "gbs_head": V * H * 2 / tm / 1e9}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", type=int, default=4, choices=[1, 4, 5])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lm-feature", action="store_true",
                    help="the trunk's LM log-prob feature on (v3_lm_feature, as in the shipped 9B checkpoint)")
    ap.add_argument("--op", default="decide",
                    choices=["decide", "gemm", "attn", "attn_state", "lm_logprob", "rows", "trunk"],
                    help="decide: the headline decision throughput; gemm / attn: operator configs 2 / 3; "
                         "attn_state: the state pass's causal attention")
    ap.add_argument("--shapes", default="", help="--op gemm: MxNxK list; --op attn: requestsxrowsxt list; "
                                                 "--op attn_state: rowsxtokens list")
    ap.add_argument("--requests", type=int, default=0, help="--op attn: requests (default 32)")
    ap.add_argument("--kernels", default="", help="--op rows: comma-separated subset of the row kernels")
    ap.add_argument("--splits", default="", help="--op gemm: comma-separated split-K counts to time per shape "
                                                 "(default: od_gemm_w8a8_plan's choice)")
    ap.add_argument("--breakdown", action="store_true", help="print per-kernel device time of one step to stderr")
    args = ap.parse_args()
    if args.op == "gemm":
        return op_gemm(args)
    if args.op == "attn":
        return op_attn(args)
    if args.op == "attn_state":
        return op_attn_state(args)
    if args.op == "lm_logprob":
        return op_lm_logprob(args)
    if args.op == "rows":
        return op_rows(args)
    if args.op == "trunk":
        return op_trunk(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch.distributed as dist
    from datetime import timedelta
    from opendecider_b200 import _lib
    from opendecider_b200 import synthetic as syn
    from opendecider_b200.backbone import Backbone
    from opendecider_b200.decider import Decider
    from opendecider_b200.distributed import DistributedDecider
    from opendecider_b200.v3 import TrunkConfig, V3Model, V3Trunk, trunk_state_dict

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg, tk, qmin, desc = workload(args.config)
    bb = Backbone.random(cfg, seed=0, device=dev, gen_device=dev)
    torch.cuda.empty_cache()
    tc = TrunkConfig(d_feat=cfg.hidden, n_feat_layers=len(cfg.feature_layers), lm_feature=args.lm_feature, **tk)
    trunk = V3Trunk(tc, trunk_state_dict(tc, seed=0), dev)
    # ONE global batch of 64 requests per GPU (weak scaling; config 5's 512 requests are the 8-GPU batch), the same on
    # every rank; each rank decides its contiguous token-balanced block (distributed.shard) and every rank gets every
    # request's probabilities back through one all_gather per step (DistributedDecider)
    reqs_all, tok = syn.decision_requests(args.config, seed=0, n_requests=64 * world)
    decider = Decider(V3Model(bb, trunk, tok, qcache_min_rows=qmin), TEMPERATURE, TEMPS)
    dd = DistributedDecider(decider) if world > 1 else None
    blocks = dd.blocks(reqs_all) if dd else [(0, len(reqs_all))]
    shapes = dd.layouts(reqs_all, blocks) if dd else None
    a_blk, b_blk = blocks[rank]
    reqs = reqs_all[a_blk:b_blk]

    def gather(probs):
        """Every rank's [probs | renorm | P(none)] block, one NCCL all_gather_into_tensor, no host sync."""
        if dd is not None:
            return dd.gather(dd.pack(*probs), shapes)
        return probs[0]

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- value: device-resident inputs (the plan uploaded once), K timed steps
    cache, items = None, None
    if args.config == 5:
        # the cached states are the workload's input (built once, untimed, with room for the appended tokens);
        # every step appends the records and decides (execute() first truncates back to the encoded length)
        appends_all = [r.append for r in reqs_all]
        appends = appends_all[a_blk:b_blk]
        n_app = len(tok([appends[0]], add_special_tokens=False)["input_ids"][0])
        cache = decider.encode_states([r.state for r in reqs], room=n_app)
        torch.cuda.synchronize()
        plan = decider.plan(reqs, cache=cache, appends=appends)
        items = lambda k: ((reqs_all, appends_all) for _ in range(k))
    else:
        plan = decider.plan(reqs)
    n_dec_local = len(plan["questions"])
    for _ in range(args.warmup):
        probs, cache = decider.execute(plan, cache)
        gather(probs)
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0, "a kernel reported a device-side error"
    barrier()
    clocks = Clocks(world) if rank == 0 else None
    _lib.GEMM_PROBE = []
    l0 = _lib.LAUNCHES[0]
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("od_timed")
    e0.record()
    for _ in range(args.steps):
        probs, cache = decider.execute(plan, cache)
        gather(probs)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    launches = (_lib.LAUNCHES[0] - l0) // max(1, args.steps)
    probe, _lib.GEMM_PROBE = _lib.GEMM_PROBE, None
    clk = clocks.stop() if clocks else None
    t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in probe)
    gemm_ops = sum(o for _, _, o, _ in probe)
    gemm_bytes = sum(b for _, _, _, b in probe)
    gemm_launches = len(probe) // max(1, args.steps)
    n_dec_total = sum(h for h, _ in shapes) if dd else n_dec_local
    decisions = n_dec_total * args.steps
    value = decisions / t_dev

    if args.breakdown and rank == 0:
        _lib.KERNEL_PROBE = {}
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        probs, cache = decider.execute(plan, cache)
        b1.record()
        torch.cuda.synchronize()
        summ = _lib.probe_summary(_lib.KERNEL_PROBE)
        _lib.KERNEL_PROBE = None
        tot = b0.elapsed_time(b1)
        for k, (n, ms) in sorted(summ.items(), key=lambda kv: -kv[1][1]):
            print(f"breakdown {k:20s} launches {n:5d}  {ms:9.2f} ms  {100 * ms / tot:5.1f} %", file=sys.stderr)
        print(f"breakdown step {tot:.2f} ms, kernels {sum(v[1] for v in summ.values()):.2f} ms", file=sys.stderr)

    # ---- e2e: the public API, one batch per step (Decider.decide_stream: tokenise + plan on the host, one pinned
    # H2D copy, kernels, the gather, one D2H read of the results, answers), batch b+1 planned while b runs
    # with N ranks: DistributedDecider.decide_stream (each rank plans and runs its block, one all_gather, and every
    # rank builds every request's answers)
    stream_in = items if items is not None else (lambda k: (reqs_all for _ in range(k)))
    cache_in = cache if items is not None else None

    def stream(k):
        if dd is not None:
            return dd.decide_stream(stream_in(k), cache=cache_in)
        return (ans for ans, _ in decider.decide_stream(stream_in(k), cache=cache_in))

    for _ in stream(1):
        pass
    torch.cuda.synchronize()
    barrier()
    h2d, d2h = decider.last_io["h2d_bytes"], decider.last_io["d2h_bytes"]
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    n_ans = 0
    for ans in stream(args.steps):
        assert len(ans) == len(reqs_all)
        n_ans += 1
    f1.record()
    torch.cuda.synchronize()
    barrier()
    t_e2e = max_over_ranks(f0.elapsed_time(f1) / 1e3)
    assert n_ans == args.steps

    if args.config == 5:
        assert plan["state"]["T"] == cache.T, "the cached plan's appended length"
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    # ---- roofline of the dominant kernel (W8A8 GEMM, int8 tensor pipe)
    peaks = {}
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
    if peaks.get("bf16_tflops_sustained"):
        peak = 2.0 * peaks["bf16_tflops_sustained"]
        peak_note = "2 x measured sustained bf16 TFLOP/s (MEASURED_PEAKS.json): the dense int8 rate is twice bf16's"
    else:
        peak = 2.0 * 1400.0
        peak_note = "2 x fallback sustained bf16 1.4 PFLOP/s"
    achieved = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
    i8 = int8_peak(dev)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        v, cores, sample, kind = cpu_baseline_sample(args.config, 20.0)
        cpu = {"value": v, "unit": "decisions/s", "cores": cores, "kind": kind,
               "sample": sample + ("; without the LM log-prob feature" if args.lm_feature else "")}
    kv_gb = sum(t.q.numel() for t in cache.k + cache.v) / 1e9 if cache is not None else 0.0
    out = {
        "metric": METRIC, "value": value, "unit": "decisions/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded random-id states, random-init weights)",
        "config": {"workload": desc + (" + LM log-prob feature" if args.lm_feature else ""),
                   "global_batch": n_dec_total, "requests": len(reqs_all), "requests_per_gpu": len(reqs),
                   "state_tokens": plan["state"]["T"],
                   "parallelism": f"dp{world}: one global batch of {len(reqs_all)} requests in contiguous "
                                  "token-balanced blocks per GPU, replicated weights, one NCCL all_gather of the "
                                  "probabilities per step",
                   "l2": f"inputs larger than L2 (7.6 GB of int8 weights and a {kv_gb:.1f} GB int8 KV cache stream "
                         "every step)"},
        "e2e": {"value": decisions / t_e2e, "unit": "decisions/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": 1e3 * t_e2e / args.steps},
        "roofline": {"bound": "tensor", "kernel": "od_gemm_w8a8 (tcgen05 kind::i8)", "achieved": achieved,
                     "peak": peak, "unit": "TOP/s (int8)", "frac": (achieved / peak) if achieved else None,
                     "peak_source": peak_note,
                     "int8_measured": i8, "frac_of_int8_sustained": (achieved / i8["sustained"]) if achieved else None,
                     "traffic": (traffic_ratio() * gemm_bytes / max(1, len(probe))) if traffic_ratio() and probe else None,
                     "traffic_unit": "DRAM bytes per launch (step average: measured DRAM / algorithmic bytes of one "
                                     "ncu launch x the algorithmic bytes of the step's launches)",
                     "traffic_source": "scaled from the committed ncu capture of one launch "
                                       "(profiles/gemm_w8a8_pair_8192x10240x4096.md); not measured in this run",
                     "launches_per_step": gemm_launches, "share_of_step": gemm_ms / 1e3 / args.steps /
                     (t_dev / args.steps) if t_dev else None},
        "cpu_baseline": cpu, "clocks": clk, "gpu_launches": launches * args.steps,
        "gpu_launches_per_step": launches}
    print(json.dumps(out))


if __name__ == "__main__":
    main()
