"""The frozen backbone of the decision forward pass on B200: a dense Qwen3.5 decoder (every layer full attention)
whose every op runs in libod_b200 (C ABI, sm_100a kernels). PyTorch only owns the buffers and the stream.

Mirrors the reference's backbone seam (src/opendecider/backbone.py): the same int8 weight layout (Int8Linear's
qweight (N, K) int8 + scale (N,) in the weight dtype, quant.py:122-127), the same int8 KV layout
(PackedCache.tensors[(layer, "keys"|"values", None)] = Int8Tensor q (S, Hkv, T, D) + scale, backbone.py:436-468), the
same LEFT-padded batched state pass (prefix_cache_batch, backbone.py:347-368) and the same positions (padded column
index; continuations start at the padded state length).

Per decoder layer (Qwen3_5DecoderLayer, modeling_qwen3_5.py:744-783) on M tokens:
    od_rmsnorm_res_quant   residual add + input RMSNorm + per-token int8         (A3/A4/A5)
    od_gemm_w8a8           fused q/k/v projection (the reference's three Int8Linear weights stacked by rows)
    od_qk_norm_rope        gated-q split, q/k RMSNorm, RoPE
    od_prefix_attn         causal / shared-prefix attention (int8 state prefix, bf16 question prefix, own keys)
    od_kv_append_i8        int8 KV cache write (state pass)                      (A6)
    od_gate_quant          o * sigmoid(gate) + per-token int8
    od_gemm_w8a8           o_proj
    od_rmsnorm_res_quant   residual add + post-attention RMSNorm + int8
    od_gemm_w8a8 SWIGLU    gate/up (rows interleaved in blocks of 128) with SiLU(gate)*up in the epilogue
    od_quant_rows_i8       per-token int8 of the MLP activation
    od_gemm_w8a8           down_proj
Stacking q/k/v (and gate/up) rows is exact: per-output-channel scales and int32 dot products of a row do not depend
on the other rows, and all three projections quantise the same normalised activation.

SmoothQuant (the reference's a8w8sq path: smooth_a8w8_ + SmoothedLinear, quant.py:317-350): a smoothed linear holds
int8(W * s) and multiplies its input by inv_s = bf16(1 / s) before the per-token quantisation. The multiply runs inside
the quantising kernel (od_rmsnorm_res_quant, od_quant_rows_i8, od_gate_quant, od_swiglu_quant). When q, k and v (or gate
and up) carry one shared vector, the stacked GEMMs run unchanged on the one smoothed activation. When their vectors
differ - the reference's calibration (scripts/smoothquant_calibrate.py) computes one per linear - each projection
quantises its own smoothed copy of the normalised activation and runs its own GEMM: q, k, v into their column ranges
of the same stacked output (od_gemm_w8a8_ld), gate and up into two outputs that od_swiglu_quant combines. Exact either
way: every smoothed input is quantised exactly as the reference quantises it.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib
from .quant import Int8Tensor, quantize_weight

GU_BLOCK = 128   # gate/up row interleave of the SwiGLU epilogue


@dataclass
class DecoderConfig:
    """Shape of a dense Qwen3.5-style GQA decoder (Qwen3_5TextConfig with every layer `full_attention`)."""
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    max_pos: int = 32768
    feature_layers: tuple = ("final",)
    dtype: torch.dtype = torch.bfloat16

    @property
    def ffn_pad(self) -> int:
        return -(-self.ffn // GU_BLOCK) * GU_BLOCK

    @property
    def qkv_out(self) -> int:
        return self.heads * self.head_dim * 2 + 2 * self.kv_heads * self.head_dim

    @classmethod
    def tiny(cls, **kw) -> "DecoderConfig":
        """4 layers, hidden 256, 4 q / 2 kv heads, head_dim 64, SwiGLU 688, vocab 1024."""
        return cls(**{**dict(vocab=1024, hidden=256, layers=4, heads=4, kv_heads=2, head_dim=64, ffn=688,
                             max_pos=4096), **kw})

    @classmethod
    def nine_b(cls, **kw) -> "DecoderConfig":
        """BASELINE configs 4/5: 36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, SwiGLU 12288, vocab 151936."""
        return cls(**{**dict(vocab=151936, hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128, ffn=12288,
                             max_pos=32768), **kw})


def hf_weight_names(cfg: DecoderConfig) -> list[tuple[str, tuple]]:
    """(name, shape) of every float weight in Qwen3_5TextModel order (the names HF's state dict uses)."""
    H, D, Hq, Hkv, F = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.ffn
    out = [("embed_tokens.weight", (cfg.vocab, H))]
    for i in range(cfg.layers):
        p = f"layers.{i}."
        out += [(p + "input_layernorm.weight", (H,)), (p + "self_attn.q_proj.weight", (Hq * D * 2, H)),
                (p + "self_attn.k_proj.weight", (Hkv * D, H)), (p + "self_attn.v_proj.weight", (Hkv * D, H)),
                (p + "self_attn.o_proj.weight", (H, Hq * D)), (p + "self_attn.q_norm.weight", (D,)),
                (p + "self_attn.k_norm.weight", (D,)), (p + "post_attention_layernorm.weight", (H,)),
                (p + "mlp.gate_proj.weight", (F, H)), (p + "mlp.up_proj.weight", (F, H)),
                (p + "mlp.down_proj.weight", (H, F))]
    out.append(("norm.weight", (H,)))
    return out


def synthetic_weights(cfg: DecoderConfig, seed: int = 0, device="cpu", layers: int | None = None) \
        -> dict[str, torch.Tensor]:
    """Random-init float weights (bf16) of the decoder, drawn in hf_weight_names order from one seeded generator:
    matrices ~ N(0, 0.02) (HF's initializer_range), RMSNorm weights ~ N(0, 0.1) (non-zero so the (1 + w) form is
    exercised; HF initialises them to 0). layers: only the embedding, the first `layers` layers and the final norm
    (for a sampled CPU baseline)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in hf_weight_names(cfg):
        if layers is not None and name.startswith("layers.") and int(name.split(".")[1]) >= layers:
            continue
        std = 0.1 if name.endswith("norm.weight") else 0.02
        out[name] = (torch.randn(*shape, generator=g, device=device) * std).to(cfg.dtype)
    return out


@dataclass
class Smooth:
    """SmoothQuant inverse scales of one decoder layer, inv_s = bf16(1 / s) per input channel (SmoothedLinear,
    quant.py:317-329); None for a linear that is not smoothed."""
    qkv: tuple               # (q_proj, k_proj, v_proj) inv_s, each (H,) or None
    gu: tuple                # (gate_proj, up_proj)
    o: torch.Tensor | None   # o_proj (Hq*D,)
    down: torch.Tensor | None  # down_proj (F_pad,): ones past F (those activations are 0)
    qkv_shared: bool = True  # one vector (or none) for q, k, v: the stacked GEMM runs on one smoothed activation
    gu_shared: bool = True


def _same(vs) -> bool:
    """True when every entry is None or all are equal tensors."""
    if all(v is None for v in vs):
        return True
    return all(v is not None for v in vs) and all(torch.equal(vs[0], v) for v in vs[1:])


@dataclass
class Layer:
    ln1: torch.Tensor
    ln2: torch.Tensor
    qkv: Int8Tensor          # (Hq*2D + 2*Hkv*D, H)
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o: Int8Tensor            # (H, Hq*D)
    gate_up: Int8Tensor | None   # (2*F_pad, H) rows interleaved in blocks of GU_BLOCK (None: separate gate / up)
    down: Int8Tensor         # (H, F_pad) columns >= F are zero
    sq: Smooth | None = None
    gate: Int8Tensor | None = None   # (F_pad, H): gate_proj alone, when gate / up are smoothed by different vectors
    up: Int8Tensor | None = None

    def qkv_parts(self, cfg: "DecoderConfig") -> list:
        """Row ranges of the stacked q/k/v weight: [(first column, Int8Tensor view)] for q_proj, k_proj, v_proj."""
        nq, nk = cfg.heads * cfg.head_dim * 2, cfg.kv_heads * cfg.head_dim
        out, c = [], 0
        for n in (nq, nk, nk):
            out.append((c, Int8Tensor(self.qkv.q[c:c + n], self.qkv.scale[c:c + n], self.qkv.dtype)))
            c += n
        return out


@dataclass
class KVCache:
    """int8 state K/V of every layer in the reference's PackedCache layout: q (S, Hkv, cap, D) int8 + scale
    (S, Hkv, cap) in the activation dtype, plus the left padding of each state (p_lo) and the padded length T <= cap
    (positions [T, cap) are room for appended tokens, invisible to attention)."""
    k: list                  # per layer Int8Tensor
    v: list
    p_lo: torch.Tensor       # (S,) int32: first real token of each state (left padding)
    T: int
    lens: list = field(default_factory=list)   # real tokens per state (CPU ints)
    kb: list | None = None   # per layer bf16 (S, Hkv, cap, D): the materialised K (prefix_attn.py:146-149), or None
    vb: list | None = None
    cap: int = 0             # capacity (the tensors' token dimension); 0 = T
    scratch: tuple | None = None   # bf16 (K, V) of one layer, (S, Hkv, cap, D): just-in-time materialisation
    enc_T: int = 0           # the encoded states' padded length and real lengths (the snapshot every append of a
    enc_lens: list = field(default_factory=list)   # decision call starts from, as PrefixCache._restore does)

    @property
    def S(self) -> int:
        return self.p_lo.numel()

    @property
    def capacity(self) -> int:
        return self.cap or self.T

    def p_hi(self) -> torch.Tensor | None:
        """(S,) int32 end of the visible prefix (= T) when the cache has room beyond T, else None (all of it)."""
        if self.capacity == self.T:
            return None
        return torch.full((self.S,), self.T, dtype=torch.int32, device=self.p_lo.device)

    def truncate(self, T: int, lens: list) -> None:
        """Forget appended tokens: back to padded length T (the K/V beyond it are overwritten by the next append)."""
        self.T, self.lens = T, list(lens)

    def rows(self, a: int, b: int) -> "KVCache":
        """View of states [a, b) (same storage)."""
        sl = lambda t: Int8Tensor(t.q[a:b], t.scale[a:b], t.dtype)
        return KVCache([sl(t) for t in self.k], [sl(t) for t in self.v], self.p_lo[a:b], self.T, self.lens[a:b],
                       [t[a:b] for t in self.kb] if self.kb is not None else None,
                       [t[a:b] for t in self.vb] if self.vb is not None else None, self.cap)

    def nbytes(self) -> int:
        return sum(t.nbytes() for t in self.k + self.v) + sum(t.nbytes for t in (self.kb or []) + (self.vb or []))


@dataclass
class PassSpec:
    """One backbone pass over R rows of t tokens (rectangular, row-major token order).
    ids/pos (R, t) on the device; own_lo/own_hi (R,) valid own-key range (None = all); prefix levels optional."""
    ids: torch.Tensor
    pos: torch.Tensor
    own_lo: torch.Tensor | None = None
    own_hi: torch.Tensor | None = None
    cache: KVCache | None = None           # level-1 int8 state prefix
    row_state: torch.Tensor | None = None  # (R,) int32 state of each row
    qkv_prefix: list | None = None         # level-2 bf16 prefix: per layer (K, V) (NQ, Lq, Hkv, D)
    row_q: torch.Tensor | None = None      # (R,) int32 question of each row
    q_len: torch.Tensor | None = None      # (NQ,) int32 real tokens of each question
    row_groups: torch.Tensor | None = None # (G, 2) int32 [first row, rows]: consecutive rows sharing state + question
    max_group_rows: int = 1
    write_cache: KVCache | None = None     # state / append pass: write this pass's K/V (rows = states) at write_t0
    write_t0: int = 0
    capture: bool = False                  # keep every layer's post-RoPE (k, v) (R, t, Hkv, D)
    features: tuple = ()                   # feature layers to return ("final" or 1-based layer numbers)
    kv_only_last: bool = False             # state pass: the last layer only needs its K/V


class Backbone:
    """Int8 weights on the device + the pass driver. Construct with from_float_weights / from_int8 / random."""

    def __init__(self, cfg: DecoderConfig, embed: Int8Tensor, layers: list, final_norm: torch.Tensor,
                 device: torch.device):
        self.cfg, self.embed, self.layers, self.final_norm, self.device = cfg, embed, layers, final_norm, device
        from .rope import rope_tables
        self.cos, self.sin = rope_tables(cfg.head_dim, cfg.rope_theta, cfg.max_pos, cfg.dtype, device)
        self.pad_id = 0
        # the state pass also writes the dequantised bf16 K/V (what materialize() gives the reference's attention,
        # prefix_attn.py:146-149) when it fits this budget, so the question / option passes stream the prefix by TMA
        # instead of dequantising it in every attention tile; 0 disables it
        total = torch.cuda.get_device_properties(device).total_memory if torch.device(device).type == "cuda" else 0
        self.materialize_budget = total // 4
        self.max_pass_tokens = 1 << 17          # state-pass chunk: 131072 tokens
        # a pass over an int8-only cache dequantises each layer's prefix once into a reused bf16 buffer when it has
        # at least this many (query token x query head) slots per state per KV head; None: never
        self.jit_min_slots = 256
        # write a pass's int8 K/V from the q/k-norm + RoPE kernel (od_qk_norm_rope_kv_i8) instead of a separate
        # od_kv_append_i8 pass: identical bytes; at the config-4 state-pass chunk (131072 tokens) 1.00 ms against
        # 0.73 + 0.44 ms for the two kernels
        self.fused_kv_write = True

    # ------------------------------------------------------------------------------------------ construction
    @classmethod
    def from_int8(cls, cfg: DecoderConfig, q: dict, norms: dict, device, inv_s: dict | None = None) -> "Backbone":
        """From the reference's int8 layout: q maps 'embed_tokens' and every 'layers.{i}.{self_attn|mlp}.{proj}' to
        (qweight int8 (N, K), scale (N,) or (N, 1)); norms maps the RMSNorm weight names to float tensors. inv_s: the
        SmoothQuant inverse scales {'layers.{i}.{self_attn|mlp}.{proj}': bf16 (K,)} of the smoothed linears, whose
        q entries then hold int8(W * s) (smooth_a8w8_, quant.py:333-350)."""
        dev = torch.device(device)
        D, F, Fp, H = cfg.head_dim, cfg.ffn, cfg.ffn_pad, cfg.hidden
        dt = cfg.dtype
        inv_s = inv_s or {}

        def qt(name):
            w, s = q[name]
            return w.to(dev).contiguous(), s.reshape(-1).to(dev, dt).contiguous()

        def iv(name, pad_to=None):
            v = inv_s.get(name)
            if v is None:
                return None
            v = v.reshape(-1).to(dev, torch.bfloat16)
            if pad_to is not None and v.numel() < pad_to:
                v = torch.cat([v, v.new_ones(pad_to - v.numel())])
            return v.contiguous()

        layers = []
        for i in range(cfg.layers):
            p = f"layers.{i}."
            parts = [qt(p + "self_attn." + n) for n in ("q_proj", "k_proj", "v_proj")]
            qkv = Int8Tensor(torch.cat([w for w, _ in parts]), torch.cat([s for _, s in parts]), dt)
            gw, gs = qt(p + "mlp.gate_proj")
            uw, us = qt(p + "mlp.up_proj")
            if Fp != F:                                   # zero rows: SiLU(0) * 0 = 0 outputs, exact padding
                gw = torch.cat([gw, gw.new_zeros(Fp - F, H)]); uw = torch.cat([uw, uw.new_zeros(Fp - F, H)])
                gs = torch.cat([gs, gs.new_ones(Fp - F)]); us = torch.cat([us, us.new_ones(Fp - F)])
            dw, ds = qt(p + "mlp.down_proj")
            if Fp != F:                                   # zero columns: the padded activations contribute 0
                dw = torch.cat([dw, dw.new_zeros(H, Fp - F)], 1)
            ow, os_ = qt(p + "self_attn.o_proj")
            sq = None
            names = [p + n for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj",
                                     "mlp.up_proj", "self_attn.o_proj", "mlp.down_proj")]
            if any(n in inv_s for n in names):
                v = [iv(n) for n in names[:6]] + [iv(names[6], Fp)]
                sq = Smooth(qkv=tuple(v[:3]), gu=tuple(v[3:5]), o=v[5], down=v[6], qkv_shared=_same(v[:3]),
                            gu_shared=_same(v[3:5]))
            layer = Layer(
                ln1=norms[p + "input_layernorm.weight"].to(dev, dt).contiguous(),
                ln2=norms[p + "post_attention_layernorm.weight"].to(dev, dt).contiguous(),
                qkv=qkv,
                q_norm=norms[p + "self_attn.q_norm.weight"].to(dev, dt).contiguous(),
                k_norm=norms[p + "self_attn.k_norm.weight"].to(dev, dt).contiguous(),
                o=Int8Tensor(ow, os_, dt), gate_up=None,
                down=Int8Tensor(dw.contiguous(), ds, dt), sq=sq)
            if sq is None or sq.gu_shared:
                gu_w = torch.stack([gw.view(Fp // GU_BLOCK, GU_BLOCK, H), uw.view(Fp // GU_BLOCK, GU_BLOCK, H)], 1)
                gu_s = torch.stack([gs.view(-1, GU_BLOCK), us.view(-1, GU_BLOCK)], 1)
                layer.gate_up = Int8Tensor(gu_w.reshape(2 * Fp, H).contiguous(), gu_s.reshape(-1).contiguous(), dt)
            else:                                         # two GEMMs on two differently smoothed activations
                layer.gate, layer.up = Int8Tensor(gw.contiguous(), gs, dt), Int8Tensor(uw.contiguous(), us, dt)
            layers.append(layer)
        ew, es = qt("embed_tokens")
        return cls(cfg, Int8Tensor(ew, es, dt), layers, norms["norm.weight"].to(dev, dt).contiguous(), dev)

    @classmethod
    def from_float_weights(cls, cfg: DecoderConfig, sd: dict, device, smooth: dict | None = None) -> "Backbone":
        """Quantise float weights exactly as the reference does at load (quantize_int8_ / Int8Embedding,
        quant.py:122-127, 186-191: per-output-row absmax int8, scale in the weight dtype), on the device.
        smooth: SmoothQuant scales s (K,) per linear, keyed as the reference's scale files key them (relative to the
        decoder's layer list: '{i}.self_attn.q_proj', ...); each such weight becomes W * s per input channel in fp32,
        stored in the weight dtype, before quantisation, and its input is multiplied by bf16(1 / s) (smooth_a8w8_ and
        SmoothedLinear, quant.py:317-350)."""
        dev = torch.device(device)
        q, norms, inv_s = {}, {}, {}
        smooth = smooth or {}
        for name, w in sd.items():
            if name.endswith("norm.weight"):
                norms[name] = w
                continue
            base = name[: -len(".weight")]
            sv = smooth.get(base[len("layers."):]) if base.startswith("layers.") else None
            w = w.to(dev)
            if sv is not None:
                sv = sv.to(dev, torch.float32)
                w = (w.float() * sv[None, :]).to(w.dtype)
                inv_s[base] = (1.0 / sv).to(torch.bfloat16)
            q[base] = quantize_weight(w)
        return cls.from_int8(cfg, q, norms, dev, inv_s)

    @classmethod
    def random(cls, cfg: DecoderConfig, seed: int = 0, device="cuda", gen_device="cpu") -> "Backbone":
        return cls.from_float_weights(cfg, synthetic_weights(cfg, seed, gen_device), device)

    # ------------------------------------------------------------------------------------------ passes
    def run(self, spec: PassSpec):
        """One pass. Returns (features (R, t, nL*H) bf16 or None, captured [(k, v)] per layer or None)."""
        cfg, dev = self.cfg, self.device
        R, t = spec.ids.shape
        M = R * t
        H, D, Hq, Hkv = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
        pos = spec.pos.reshape(-1).to(torch.int32).contiguous()
        x = _lib.embed_i8(spec.ids.reshape(-1), self.embed.q, self.embed.scale)     # (M, H): layer 0 input
        r = x                                                                          # residual stream
        feats = {}
        want = [f for f in spec.features]
        captured = [] if spec.capture else None
        d = None
        cache = spec.cache
        p_hi = cache.p_hi() if cache is not None else None
        # dequantise the prefix once per layer (into a reused bf16 buffer) when the whole-cache copy was not kept
        # and the pass has at least two 128-slot query tiles per state (each would otherwise dequantise it again)
        jit = cache is not None and cache.kb is None and self.jit_min_slots is not None and \
            (M // max(1, cache.S)) * (Hq // Hkv) >= self.jit_min_slots and \
            self.jit_bytes(cache) <= self.materialize_budget
        for li, L in enumerate(self.layers):
            last = li == cfg.layers - 1
            sq = L.sq
            nk = {} if li == 0 else dict(res_in=r, res_out=r)
            if sq is None or sq.qkv_shared:
                hq, hs = _lib.rmsnorm_res_quant(r if li == 0 else d, L.ln1, cfg.eps,
                                                inv_s=sq.qkv[0] if sq is not None else None, **nk)
                qkv = _lib.gemm_w8a8(hq, hs, L.qkv.q, L.qkv.scale, _lib.OD_EPI_BF16)
            else:                                           # q, k, v smoothed by different vectors
                y = torch.empty(M, H, dtype=cfg.dtype, device=dev)
                _lib.rmsnorm_res_quant(r if li == 0 else d, L.ln1, cfg.eps, y_out=y, want_q=False, **nk)
                qkv = torch.empty(M, cfg.qkv_out, dtype=cfg.dtype, device=dev)
                for (c, W), inv in zip(L.qkv_parts(cfg), sq.qkv):
                    xq, xs = _lib.quant_rows(y, scale_dtype=torch.float32, inv_s=inv)
                    _lib.gemm_w8a8(xq, xs.view(-1), W.q, W.scale, _lib.OD_EPI_BF16,
                                   out=qkv[:, c:c + W.q.shape[0]])
            if li > 0 and li in want:                       # output of decoder layer li (1-based feature number)
                feats[li] = r.clone()
            wc = spec.write_cache
            if wc is not None and self.fused_kv_write and cfg.dtype == torch.bfloat16:
                # the pass's K/V go into the int8 cache (and its kept bf16 copy) from the same kernel
                q, k, v = _lib.qk_norm_rope_kv(qkv, pos, self.cos, self.sin, L.q_norm, L.k_norm, cfg.eps, Hq, Hkv, D,
                                               t, wc.k[li].q, wc.v[li].q, wc.k[li].scale, wc.v[li].scale,
                                               spec.write_t0, kb=wc.kb[li] if wc.kb is not None else None,
                                               vb=wc.vb[li] if wc.vb is not None else None)
            else:
                q, k, v = _lib.qk_norm_rope(qkv, pos, self.cos, self.sin, L.q_norm, L.k_norm, cfg.eps, Hq, Hkv, D)
                if wc is not None:
                    _lib.kv_append(k.view(R, t, Hkv, D), v.view(R, t, Hkv, D), wc.k[li].q, wc.v[li].q,
                                   wc.k[li].scale, wc.v[li].scale, t0=spec.write_t0,
                                   kb=wc.kb[li] if wc.kb is not None else None,
                                   vb=wc.vb[li] if wc.vb is not None else None)
            k4, v4 = k.view(R, t, Hkv, D), v.view(R, t, Hkv, D)
            if captured is not None:
                captured.append((k4, v4))
            if last and spec.kv_only_last:
                break
            Kb = Vb = None
            if cache is not None and cache.kb is not None:
                Kb, Vb = cache.kb[li], cache.vb[li]
            elif cache is not None and jit:                 # this layer's cache materialised just for this pass
                Kb, Vb = self._materialise_layer(cache, li)
            o = _lib.prefix_attn(
                q.view(R, t, Hq, D), k4, v4, D ** -0.5,
                Kp=(Kb if Kb is not None else cache.k[li].q) if cache else None,
                Vp=(Vb if Vb is not None else cache.v[li].q) if cache else None,
                ksc=cache.k[li].scale if cache and Kb is None else None,
                vsc=cache.v[li].scale if cache and Kb is None else None,
                row_state=spec.row_state, p_lo=cache.p_lo if cache else None, p_hi=p_hi,
                Kq=spec.qkv_prefix[li][0] if spec.qkv_prefix else None,
                Vq=spec.qkv_prefix[li][1] if spec.qkv_prefix else None, row_q=spec.row_q, q_len=spec.q_len,
                own_lo=spec.own_lo, own_hi=spec.own_hi, row_groups=spec.row_groups,
                max_group_rows=spec.max_group_rows)
            oq, os_ = _lib.gate_quant(o.view(M, Hq * D), qkv, Hq, D, inv_s=sq.o if sq is not None else None)
            a = _lib.gemm_w8a8(oq, os_, L.o.q, L.o.scale, _lib.OD_EPI_BF16)
            if L.gate_up is not None:
                mq, ms = _lib.rmsnorm_res_quant(a, L.ln2, cfg.eps, res_in=r, res_out=r,
                                                inv_s=sq.gu[0] if sq is not None else None)
                hm = _lib.gemm_w8a8(mq, ms, L.gate_up.q, L.gate_up.scale, _lib.OD_EPI_SWIGLU)
                dq, dsc = _lib.quant_rows(hm, scale_dtype=torch.float32, inv_s=sq.down if sq is not None else None)
            else:                                           # gate and up smoothed by different vectors
                y2 = torch.empty(M, H, dtype=cfg.dtype, device=dev)
                _lib.rmsnorm_res_quant(a, L.ln2, cfg.eps, res_in=r, res_out=r, y_out=y2, want_q=False)
                gq, gs = _lib.quant_rows(y2, scale_dtype=torch.float32, inv_s=sq.gu[0])
                g = _lib.gemm_w8a8(gq, gs.view(-1), L.gate.q, L.gate.scale, _lib.OD_EPI_BF16)
                uq, us = _lib.quant_rows(y2, scale_dtype=torch.float32, inv_s=sq.gu[1])
                u = _lib.gemm_w8a8(uq, us.view(-1), L.up.q, L.up.scale, _lib.OD_EPI_BF16)
                dq, dsc = _lib.swiglu_quant(g, u, inv_s=sq.down)
            d = _lib.gemm_w8a8(dq, dsc.view(-1), L.down.q, L.down.scale, _lib.OD_EPI_BF16)
        out = None
        if want and not spec.kv_only_last:
            y = torch.empty(M, H, dtype=cfg.dtype, device=dev)
            _lib.rmsnorm_res_quant(d, self.final_norm, cfg.eps, res_in=r, res_out=r, y_out=y, want_q=False)
            if cfg.layers in want:
                feats[cfg.layers] = r
            feats["final"] = y
            out = torch.cat([feats[f if f == "final" else int(f)].view(R, t, H) for f in want], -1)
        return out, captured

    # ------------------------------------------------------------------------------------------ state pass
    def new_cache(self, S: int, T: int, cap: int | None = None) -> KVCache:
        """Empty cache for S states of padded length T, with room for tokens up to `cap` (default T)."""
        cfg, dev = self.cfg, self.device
        C = max(T, cap or T)
        mk = lambda: Int8Tensor(torch.empty(S, cfg.kv_heads, C, cfg.head_dim, dtype=torch.int8, device=dev),
                                torch.empty(S, cfg.kv_heads, C, dtype=cfg.dtype, device=dev), cfg.dtype)
        cache = KVCache([mk() for _ in range(cfg.layers)], [mk() for _ in range(cfg.layers)],
                        torch.zeros(S, dtype=torch.int32, device=dev), T, cap=C)
        bf16_bytes = 2 * cfg.layers * S * cfg.kv_heads * C * cfg.head_dim * 2
        if cfg.dtype == torch.bfloat16 and 0 < bf16_bytes <= self.materialize_budget:
            mb = lambda: torch.empty(S, cfg.kv_heads, C, cfg.head_dim, dtype=torch.bfloat16, device=dev)
            cache.kb = [mb() for _ in range(cfg.layers)]
            cache.vb = [mb() for _ in range(cfg.layers)]
        return cache

    def jit_bytes(self, cache: KVCache) -> int:
        """bytes of one layer's bf16 K and V (the just-in-time materialisation buffer)."""
        return 2 * cache.S * self.cfg.kv_heads * cache.capacity * self.cfg.head_dim * 2

    def _materialise_layer(self, cache: KVCache, li: int):
        """bf16(q * s) of layer li's cached K and V into the cache's reused buffer (exactly what the in-kernel
        dequantisation and materialize() compute)."""
        if cache.scratch is None:
            shp = (cache.S, self.cfg.kv_heads, cache.capacity, self.cfg.head_dim)
            cache.scratch = (torch.empty(shp, dtype=torch.bfloat16, device=self.device),
                             torch.empty(shp, dtype=torch.bfloat16, device=self.device))
        D = self.cfg.head_dim
        Kb, Vb = cache.scratch
        _lib.dequant_rows(cache.k[li].q.view(-1, D), cache.k[li].scale.view(-1, 1), torch.bfloat16, out=Kb.view(-1, D))
        _lib.dequant_rows(cache.v[li].q.view(-1, D), cache.v[li].scale.view(-1, 1), torch.bfloat16, out=Vb.view(-1, D))
        return Kb, Vb

    def plan_state(self, seqs, up=None) -> dict:
        """Host layout of the batched state pass (Backbone.prefix_cache_batch, backbone.py:347-368): states LEFT-padded
        to the longest, positions = padded column index, uploaded once."""
        lens = [len(s) for s in seqs]
        S, T = len(seqs), max(lens)
        ids = torch.tensor([[self.pad_id] * (T - n) + list(s) for s, n in zip(seqs, lens)], dtype=torch.long)
        pad = torch.tensor([T - n for n in lens], dtype=torch.int32)
        pos = torch.arange(T, dtype=torch.int32).expand(S, T).contiguous()
        up = up or (lambda x: x.to(self.device, non_blocking=True))
        return {"S": S, "T": T, "lens": lens, "ids": up(ids), "pos": up(pos), "pad": up(pad)}

    def run_state(self, plan: dict, cache: KVCache | None = None) -> KVCache:
        """ONE pass over all states; every layer's int8 K/V is written by od_kv_append_i8 (PackedCache.pack's
        Int8Tensor.quantize, backbone.py:446). The last layer stops after its K/V projection: nothing downstream
        reads its attention or MLP output (the state pass keeps no hidden states, v3.py:317)."""
        S, T = plan["S"], plan["T"]
        cap = max(T, plan.get("cap") or T)
        if cache is None or cache.S != S or cache.capacity != cap:
            cache = self.new_cache(S, T, cap)
        cache.T = cache.enc_T = T
        cache.p_lo.copy_(plan["pad"])
        cache.lens, cache.enc_lens = list(plan["lens"]), list(plan["lens"])
        # states in chunks of at most `max_pass_tokens` tokens (bounded activation memory), each written into its
        # rows of the cache
        per = max(1, self.max_pass_tokens // max(1, T))
        for a in range(0, S, per):
            b = min(S, a + per)
            self.run(PassSpec(ids=plan["ids"][a:b], pos=plan["pos"][a:b], own_lo=plan["pad"][a:b],
                              write_cache=cache.rows(a, b), kv_only_last=True))
        return cache

    def run_append(self, ids: torch.Tensor, cache: KVCache) -> KVCache:
        """PrefixCache.encode's continuation (state_cache.py:140-146) for every state at once: n new tokens per state
        (ids (S, n) on the device) at positions T .. T+n-1 attend the cached prefix [p_lo, T) and each other causally;
        their int8 K/V (Int8Tensor.quantize, the snapshot's quantisation) are written at [T, T+n). Advances T."""
        S, n = ids.shape
        assert S == cache.S and cache.T + n <= cache.capacity, "append: cache rows / capacity"
        T = cache.T
        pos = (T + torch.arange(n, device=ids.device, dtype=torch.int32)).expand(S, n).contiguous()
        rows = torch.arange(S, device=ids.device, dtype=torch.int32)
        self.run(PassSpec(ids=ids, pos=pos, cache=cache, row_state=rows, write_cache=cache, write_t0=T,
                          kv_only_last=True))
        cache.T = T + n
        cache.lens = [l + n for l in cache.lens]
        return cache

    def token_logprob(self, h: torch.Tensor, tok: torch.Tensor) -> torch.Tensor:
        """Backbone.token_logprob (backbone.py:165-178) with the tied int8 head: log softmax(h W^T)[tok] for h (M, H)
        bf16 and tok (M,) int64 -> (M,) fp32 (od_lm_logprob). The head's bf16 rows (head_rows(): bf16(q * s)) are
        materialised once and kept."""
        if getattr(self, "_head_bf16", None) is None:
            q, sc = self.embed.q, self.embed.scale
            self._head_bf16 = _lib.dequant_rows(q, sc.reshape(-1, 1), torch.bfloat16)
        return _lib.lm_logprob(h, self._head_bf16, self.embed.q, self.embed.scale.reshape(-1), tok)

    def prefix_cache_batch(self, seqs) -> KVCache:
        """Backbone.prefix_cache_batch (backbone.py:347-368) on B200: returns the int8 KV cache of all states."""
        return self.run_state(self.plan_state(seqs))
