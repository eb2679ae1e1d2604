"""ctypes binding of libod_b200.so (the C ABI declared in include/od_b200.h) and thin tensor-level wrappers.

The library is the only implementation of the hot path: there is no CPU or PyTorch fallback. Loading fails loudly
when the shared object is missing (build it with `python -m opendecider_b200.build`), and every wrapper raises
ODError with the library's own message when a call returns a non-zero status. Wrappers launch on PyTorch's current
CUDA stream and never synchronise.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_int64, c_uint8, c_void_p

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libod_b200.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "od_b200.h")

OD_BF16, OD_F16, OD_F32 = 0, 1, 2
OD_EPI_BF16, OD_EPI_SWIGLU, OD_EPI_INT32 = 0, 1, 2
OD_TRUNK_SELF, OD_TRUNK_KEYS, OD_TRUNK_CLS = 0, 1, 2
_DT = {torch.bfloat16: OD_BF16, torch.float16: OD_F16, torch.float32: OD_F32}


class ODError(RuntimeError):
    """A libod_b200 call returned an error status."""


class AttnDims(ctypes.Structure):
    _fields_ = [("R", c_int64), ("t", c_int64), ("S", c_int64), ("T", c_int64), ("NQ", c_int64), ("Lq", c_int64),
                ("Hq", c_int), ("Hkv", c_int), ("D", c_int), ("scale_dtype", c_int), ("sm_scale", c_float),
                ("G", c_int64), ("max_group_rows", c_int), ("prefix_bf16", c_int),
                ("nsplit", c_int)]


# exported symbol -> argument types (the declarations of include/od_b200.h)
SIGNATURES = {
    "od_last_error": [],
    "od_version": [],
    "od_device_error": [c_void_p, POINTER(c_int32)],
    "od_selftest_bounded_wait": [c_int64, c_void_p],
    "od_quant_rows_i8": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int, c_void_p],
    "od_dequant_rows_i8": [c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_int, c_void_p],
    "od_kv_append_i8": [c_void_p, c_void_p, c_int, c_int64, c_int64, c_int, c_int, c_int64, c_int64, c_int64,
                        c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                        c_int64, c_int64, c_void_p],
    "od_rmsnorm_res_quant": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int64, c_int, c_void_p,
                             c_void_p, c_void_p, c_void_p],
    "od_gemm_w8a8": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p],
    "od_gemm_w8a8_ld": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_int64,
                        c_void_p],
    "od_gemm_w8a8_plan": [c_int64, c_int64, c_int64, c_int, POINTER(c_int), POINTER(c_int64)],
    "od_gemm_w8a8_splitk": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                            c_int64, c_int, c_void_p, c_int64, c_void_p],
    "od_embed_i8": [c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p],
    "od_qk_norm_rope": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_int64, c_int,
                        c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "od_qk_norm_rope_kv_i8": [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float, c_int64,
                              c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p],
    "od_gate_quant": [c_void_p, c_void_p, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "od_swiglu_quant": [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p],
    "od_prefix_attn": [c_void_p] * 20 + [AttnDims, c_void_p, c_int64, c_void_p],
    "od_prefix_attn_plan": [POINTER(AttnDims), c_int, POINTER(c_int), POINTER(c_int64)],
    "od_prefix_attn_noalloc": [c_void_p] * 20 + [AttnDims, c_void_p],
    "od_lm_logprob_plan": [c_int64, c_int64, c_int, POINTER(c_int), POINTER(c_int64)],
    "od_lm_logprob": [c_void_p, c_int64, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                      c_int64, c_int, c_void_p],
    "od_readout": [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                   c_void_p],
    "od_split_tf32": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p],
    "od_scalenorm_split": [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_float, c_void_p,
                           c_void_p, c_int64, c_void_p],
    "od_gemm_f32": [c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                    c_void_p, c_void_p, c_int, c_int, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p],
    "od_xatglu_split": [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64, c_void_p],
    "od_trunk_attn": [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                      c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_int, c_void_p, c_void_p, c_void_p,
                      c_int64, c_void_p],
}

_lib = None

# kernel launches issued through this module (every compute wrapper launches exactly one kernel)
LAUNCHES = [0]
# optional per-launch timing of od_gemm_w8a8: a list that receives (start event, end event, int ops) per launch
GEMM_PROBE: list | None = None
# optional per-launch timing of every wrapper: dict name -> list of (start event, end event)
KERNEL_PROBE: dict | None = None


def _probed(fn):
    """Record CUDA events around a wrapper's launch when KERNEL_PROBE is set (diagnostics; off by default)."""
    import functools

    @functools.wraps(fn)
    def w(*a, **k):
        probe = KERNEL_PROBE
        if probe is None:
            return fn(*a, **k)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = fn(*a, **k)
        e1.record()
        probe.setdefault(fn.__name__, []).append((e0, e1))
        return out
    return w


def probe_summary(probe: dict) -> dict:
    """{wrapper: (launches, total ms)} of a KERNEL_PROBE after synchronisation."""
    return {k: (len(v), sum(a.elapsed_time(b) for a, b in v)) for k, v in probe.items()}


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library once (raises if it is missing: the product has no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise ODError(f"{path} is missing: build it with `python -m opendecider_b200.build` (no fallback path)")
        lib = ctypes.CDLL(path)
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name in ("od_last_error", "od_version") else c_int
        _lib = lib
    return _lib


def _check(rc: int, what: str) -> None:
    LAUNCHES[0] += 1
    if rc != 0:
        msg = load().od_last_error().decode(errors="replace")
        raise ODError(f"{what}: status {rc}: {msg}")


def _p(t: torch.Tensor | None):
    return None if t is None else c_void_p(t.data_ptr())


def _stream(device: torch.device) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts: torch.Tensor | None) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ODError("libod_b200 kernels take CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
    return dev


def device_error(device: torch.device | None = None) -> int:
    """Reads and clears the device-side error word (bounded waits that gave up, out-of-range ids). Synchronises."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    v = c_int32(0)
    rc = load().od_device_error(_stream(device), ctypes.byref(v))
    if rc != 0:
        raise ODError(f"od_device_error: status {rc}: {load().od_last_error().decode(errors='replace')}")
    return v.value


# ------------------------------------------------------------------------------------------------ wrappers
@_probed
def quant_rows(x: torch.Tensor, scale_dtype: torch.dtype | None = None, inv_s: torch.Tensor | None = None,
               q: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """Int8Tensor.quantize over the last dim of a 2-D (row-strided) tensor: returns (q int8 (M, K), scale (M, 1))."""
    dev = _need_cuda(x, inv_s)
    assert x.dim() == 2 and x.stride(1) == 1, "x must be (M, K) with a contiguous last dim"
    M, K = x.shape
    sdt = scale_dtype or (x.dtype if x.dtype != torch.float32 else torch.float32)
    q = torch.empty(M, K, dtype=torch.int8, device=dev) if q is None else q
    scale = torch.empty(M, 1, dtype=sdt, device=dev) if scale is None else scale
    _check(load().od_quant_rows_i8(_p(x), _DT[x.dtype], M, K, x.stride(0), _p(inv_s), _p(q), _p(scale), _DT[sdt],
                                   _stream(dev)), "od_quant_rows_i8")
    return q, scale


@_probed
def dequant_rows(q: torch.Tensor, scale: torch.Tensor, out_dtype: torch.dtype, out: torch.Tensor | None = None):
    """Int8Tensor.dequantize: bf16/f16/f32 (q * scale) per row of the last dim; into `out` when given."""
    dev = _need_cuda(q, scale)
    M, K = q.reshape(-1, q.shape[-1]).shape
    y = torch.empty(q.shape, dtype=out_dtype, device=dev) if out is None else out
    assert y.dtype == out_dtype and y.numel() == q.numel() and y.is_contiguous()
    _check(load().od_dequant_rows_i8(_p(q), _p(scale), _DT[scale.dtype], M, K, _p(y), _DT[out_dtype], _stream(dev)),
           "od_dequant_rows_i8")
    return y


@_probed
def kv_append(k: torch.Tensor, v: torch.Tensor, kq: torch.Tensor, vq: torch.Tensor, ksc: torch.Tensor,
              vsc: torch.Tensor, t0: int, kb: torch.Tensor | None = None, vb: torch.Tensor | None = None) -> None:
    """Quantise new keys/values k, v (S, t, Hkv, D) (any strides, last dim contiguous) into the int8 cache
    kq/vq (S, Hkv, T_cap, D) + ksc/vsc (S, Hkv, T_cap) at token offset t0; kb/vb (same shape as kq, dtype of k):
    the materialised copy of the cache, extended with the same rows."""
    dev = _need_cuda(k, v, kq, vq, ksc, vsc)
    S, t, Hkv, D = k.shape
    assert k.stride(3) == 1 and v.stride(3) == 1 and kq.is_contiguous() and vq.is_contiguous()
    assert ksc.dtype == k.dtype and vsc.dtype == v.dtype and k.dtype == v.dtype
    assert (kb is None) == (vb is None)
    if kb is not None:
        assert kb.shape == kq.shape and vb.shape == vq.shape and kb.is_contiguous() and vb.is_contiguous()
        assert kb.dtype == k.dtype and vb.dtype == k.dtype
    _check(load().od_kv_append_i8(_p(k), _p(v), _DT[k.dtype], S, t, Hkv, D, k.stride(0), k.stride(1), k.stride(2),
                                  v.stride(0), v.stride(1), v.stride(2), _p(kq), _p(vq), _p(ksc), _p(vsc),
                                  _p(kb), _p(vb),
                                  kq.shape[2], t0, _stream(dev)), "od_kv_append_i8")


@_probed
def rmsnorm_res_quant(x: torch.Tensor, w: torch.Tensor, eps: float, res_in: torch.Tensor | None = None,
                      res_out: torch.Tensor | None = None, inv_s: torch.Tensor | None = None,
                      y_out: torch.Tensor | None = None, want_q: bool = True, q: torch.Tensor | None = None,
                      s: torch.Tensor | None = None):
    """Residual add + RMSNorm (1+w) + optional smoothing + per-token int8. Returns (q, s) (or (None, None))."""
    dev = _need_cuda(x, w, res_in, inv_s)
    M, H = x.shape
    if want_q:
        q = torch.empty(M, H, dtype=torch.int8, device=dev) if q is None else q
        s = torch.empty(M, dtype=torch.float32, device=dev) if s is None else s
    _check(load().od_rmsnorm_res_quant(_p(x), _p(res_in), _p(res_out), _p(w), _p(inv_s), eps, M, H, _p(y_out),
                                       _p(q) if want_q else None, _p(s) if want_q else None, _stream(dev)),
           "od_rmsnorm_res_quant")
    return (q, s) if want_q else (None, None)


_GEMM_PLANS: dict = {}
_SPLITK_WS: dict = {}


def _gemm_plan(M: int, N: int, K: int, dev) -> int:
    """od_gemm_w8a8_plan's split count for this shape on this GPU (cached per shape)."""
    key = (M, N, K, dev.index)
    if key not in _GEMM_PLANS:
        n, b = ctypes.c_int(1), ctypes.c_int64(0)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        _check(load().od_gemm_w8a8_plan(M, N, K, sms, ctypes.byref(n), ctypes.byref(b)), "od_gemm_w8a8_plan")
        _GEMM_PLANS[key] = n.value
    return _GEMM_PLANS[key]


def _splitk_bytes(M: int, N: int, splits: int) -> int:
    tiles = -(-M // 128) * -(-N // 256)
    return tiles * splits * 128 * 256 * 4


def _splitk_workspace(dev, nbytes: int) -> torch.Tensor:
    """The split-K partials' workspace of a device (grown on demand). Calls are stream-ordered on the device's current
    stream, so two never use it at the same time."""
    ws = _SPLITK_WS.get(dev.index)
    if ws is None or ws.numel() * 4 < nbytes:
        ws = torch.empty(-(-nbytes // 4), dtype=torch.int32, device=dev)
        _SPLITK_WS[dev.index] = ws
    return ws


@_probed
def gemm_w8a8(a: torch.Tensor, sa: torch.Tensor | None, w: torch.Tensor, sw: torch.Tensor | None,
              epilogue: int = OD_EPI_BF16, out: torch.Tensor | None = None, splits: int | None = None) -> torch.Tensor:
    """int8 (M, K) x int8 (N, K)^T on tcgen05: bf16 (M, N) / SwiGLU bf16 (M, N/2) / int32 (M, N). `out` may be a
    column slice of a wider row-major buffer (its row stride is passed as the output leading dimension). splits: the
    K range split over work items for small M (None: od_gemm_w8a8_plan's choice; 1: none)."""
    dev = _need_cuda(a, w, sa, sw)
    M, K = a.shape
    N = w.shape[0]
    if out is None:
        if epilogue == OD_EPI_INT32:
            out = torch.empty(M, N, dtype=torch.int32, device=dev)
        elif epilogue == OD_EPI_SWIGLU:
            out = torch.empty(M, N // 2, dtype=torch.bfloat16, device=dev)
        else:
            out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    probe = GEMM_PROBE
    if probe is not None:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    assert out.dim() == 2 and out.stride(1) == 1 and out.shape[0] == M, "out: (M, cols) with contiguous rows"
    if splits is None:
        splits = _gemm_plan(M, N, K, dev)
    if splits > 1:                                  # small M: the K range split over CTAs (exact int32 sums)
        ws = _splitk_workspace(dev, _splitk_bytes(M, N, splits))
        _check(load().od_gemm_w8a8_splitk(_p(a), _p(sa), _p(w), _p(sw), _p(out), M, N, K, epilogue, out.stride(0),
                                          splits, _p(ws), ws.numel() * 4, _stream(dev)), "od_gemm_w8a8")
    else:
        _check(load().od_gemm_w8a8_ld(_p(a), _p(sa), _p(w), _p(sw), _p(out), M, N, K, epilogue, out.stride(0),
                                      _stream(dev)), "od_gemm_w8a8")
    if probe is not None:
        e1.record()
        probe.append((e0, e1, 2 * M * N * K, M * K + N * K + out.numel() * out.element_size() + 4 * M + 2 * N))
    return out


@_probed
def embed_i8(ids: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, out: torch.Tensor | None = None):
    dev = _need_cuda(ids, qweight, scale)
    ids = ids.reshape(-1).to(torch.int64).contiguous()
    V, H = qweight.shape
    out = torch.empty(ids.numel(), H, dtype=torch.bfloat16, device=dev) if out is None else out
    _check(load().od_embed_i8(_p(ids), ids.numel(), _p(qweight), _p(scale), V, H, _p(out), _stream(dev)),
           "od_embed_i8")
    return out


@_probed
def qk_norm_rope(qkv: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, qnorm_w: torch.Tensor,
                 knorm_w: torch.Tensor, eps: float, Hq: int, Hkv: int, D: int, q_out=None, k_out=None, v_out=None):
    dev = _need_cuda(qkv, pos, cos, sin)
    M = qkv.shape[0]
    q_out = torch.empty(M, Hq, D, dtype=torch.bfloat16, device=dev) if q_out is None else q_out
    k_out = torch.empty(M, Hkv, D, dtype=torch.bfloat16, device=dev) if k_out is None else k_out
    v_out = torch.empty(M, Hkv, D, dtype=torch.bfloat16, device=dev) if v_out is None else v_out
    _check(load().od_qk_norm_rope(_p(qkv), _p(pos), _p(cos), _p(sin), cos.shape[0], _p(qnorm_w), _p(knorm_w), eps, M,
                                  Hq, Hkv, D, _p(q_out), _p(k_out), _p(v_out), _stream(dev)), "od_qk_norm_rope")
    return q_out, k_out, v_out


@_probed
def qk_norm_rope_kv(qkv: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                    qnorm_w: torch.Tensor, knorm_w: torch.Tensor, eps: float, Hq: int, Hkv: int, D: int, t: int,
                    kq: torch.Tensor, vq: torch.Tensor, ksc: torch.Tensor, vsc: torch.Tensor, t0: int,
                    kb: torch.Tensor | None = None, vb: torch.Tensor | None = None):
    """qk_norm_rope plus the int8 cache write of the pass's K/V (kv_append's bytes): the M = S x t tokens are rows of
    t tokens, row r written at positions t0 .. t0 + t - 1 of state r of kq/vq (S, Hkv, T_cap, D) + ksc/vsc; kb/vb:
    the materialised bf16 copy. Returns (q, k, v) as qk_norm_rope."""
    dev = _need_cuda(qkv, pos, cos, sin, kq, vq, ksc, vsc)
    M = qkv.shape[0]
    assert kq.is_contiguous() and vq.is_contiguous() and ksc.dtype == torch.bfloat16 and vsc.dtype == torch.bfloat16
    assert (kb is None) == (vb is None) and kq.shape[0] * t == M
    q_out = torch.empty(M, Hq, D, dtype=torch.bfloat16, device=dev)
    k_out = torch.empty(M, Hkv, D, dtype=torch.bfloat16, device=dev)
    v_out = torch.empty(M, Hkv, D, dtype=torch.bfloat16, device=dev)
    _check(load().od_qk_norm_rope_kv_i8(_p(qkv), _p(pos), _p(cos), _p(sin), cos.shape[0], _p(qnorm_w), _p(knorm_w),
                                        eps, M, Hq, Hkv, D, _p(q_out), _p(k_out), _p(v_out), t, _p(kq), _p(vq),
                                        _p(ksc), _p(vsc), _p(kb), _p(vb), kq.shape[2], t0, _stream(dev)),
           "od_qk_norm_rope_kv_i8")
    return q_out, k_out, v_out


@_probed
def gate_quant(o: torch.Tensor, qkv: torch.Tensor, Hq: int, D: int, q=None, s=None, inv_s=None):
    """bf16(o * bf16(sigmoid(gate))) [x inv_s, the o_proj SmoothedLinear] -> per-token int8 q (M, Hq*D), fp32 s (M,)."""
    dev = _need_cuda(o, qkv, inv_s)
    M = o.shape[0]
    q = torch.empty(M, Hq * D, dtype=torch.int8, device=dev) if q is None else q
    s = torch.empty(M, dtype=torch.float32, device=dev) if s is None else s
    _check(load().od_gate_quant(_p(o), _p(qkv), qkv.stride(0), M, Hq, D, _p(inv_s), _p(q), _p(s), _stream(dev)),
           "od_gate_quant")
    return q, s


@_probed
def swiglu_quant(g: torch.Tensor, u: torch.Tensor, inv_s: torch.Tensor | None = None, q=None, s=None):
    """bf16(bf16(silu(g)) * u) [x inv_s, the down_proj SmoothedLinear] -> per-token int8 q (M, F), fp32 s (M,):
    the MLP of a layer whose gate_proj and up_proj are smoothed by different vectors (two GEMMs)."""
    dev = _need_cuda(g, u, inv_s)
    assert g.shape == u.shape and g.is_contiguous() and u.is_contiguous()
    M, F = g.shape
    q = torch.empty(M, F, dtype=torch.int8, device=dev) if q is None else q
    s = torch.empty(M, dtype=torch.float32, device=dev) if s is None else s
    _check(load().od_swiglu_quant(_p(g), _p(u), M, F, _p(inv_s), _p(q), _p(s), _stream(dev)), "od_swiglu_quant")
    return q, s


# query slots one od_prefix_attn CTA holds (two 128-slot tensor-core tiles): a row group may fill it
ATTN_CTA_SLOTS = 256
_PLANS: dict = {}


def _attn_plan(dims: AttnDims, dev) -> tuple[int, int]:
    """od_prefix_attn_plan for this GPU's SM count, cached per shape."""
    key = (dev.index, dims.R, dims.t, dims.S, dims.T, dims.Hq, dims.Hkv, dims.D, dims.G, dims.max_group_rows,
           dims.prefix_bf16)
    got = _PLANS.get(key)
    if got is None:
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        n, b = ctypes.c_int(1), ctypes.c_int64(0)
        _check(load().od_prefix_attn_plan(ctypes.byref(dims), sms, ctypes.byref(n), ctypes.byref(b)),
               "od_prefix_attn_plan")
        got = _PLANS[key] = (n.value, b.value)
    return got


@_probed
def prefix_attn(q: torch.Tensor, k_own: torch.Tensor, v_own: torch.Tensor, sm_scale: float, *,
                Kp=None, Vp=None, ksc=None, vsc=None, row_state=None, p_lo=None, p_hi=None, pmask=None,
                Kq=None, Vq=None, row_q=None, q_len=None, own_lo=None, own_hi=None, row_groups=None,
                max_group_rows: int = 1, out=None, want_lse: bool = False, nsplit: int | None = None):
    """q (R, t, Hq, D), own k/v (R, t, Hkv, D) bf16; state prefix Kp/Vp (S, Hkv, T, D): int8 + scales ksc/vsc
    (S, Hkv, T[, 1]), or bf16 (the materialised cache, scales unused);
    optional bf16 question prefix Kq/Vq (NQ, Lq, Hkv, D); own keys valid in [own_lo[r], own_hi[r]) and causal;
    row_groups (G, 2) int32 [first row, rows] of consecutive rows sharing state and question, processed together
    (max_group_rows = the largest). nsplit: CTAs per state prefix (None: od_prefix_attn_plan's choice for this
    GPU; the partial results then merge in a second kernel through a workspace from torch's allocator).
    Returns o (R, t, Hq, D) [, lse (R, Hq, t)]."""
    dev = _need_cuda(q, k_own, v_own, Kp, Kq)
    R, t, Hq, D = q.shape
    Hkv = k_own.shape[2]
    out = torch.empty_like(q) if out is None else out
    lse = torch.empty(R, Hq, t, dtype=torch.float32, device=dev) if want_lse else None
    S, T = (Kp.shape[0], Kp.shape[2]) if Kp is not None else (0, 0)
    NQ, Lq = (Kq.shape[0], Kq.shape[1]) if Kq is not None else (0, 0)
    pbf16 = Kp is not None and Kp.dtype == torch.bfloat16
    assert Kp is None or pbf16 or Kp.dtype == torch.int8, "the state prefix is int8 (+ scales) or bf16"
    sdt = _DT[ksc.dtype] if (ksc is not None and not pbf16) else OD_BF16
    G = row_groups.shape[0] if row_groups is not None else R
    dims = AttnDims(R, t, S, T, NQ, Lq, Hq, Hkv, D, sdt, sm_scale, G, max_group_rows if row_groups is not None else 1,
                    1 if pbf16 else 0, 0)
    ws, ws_bytes = None, 0
    if Kp is not None:
        if nsplit is None:
            nsplit, ws_bytes = _attn_plan(dims, dev)
        else:
            ws_bytes = 4 * nsplit * R * t * Hq * (D + 1) if nsplit > 1 else 0
        dims.nsplit = nsplit
        if nsplit > 1:
            ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device=dev)
    _check(load().od_prefix_attn(_p(q), _p(Kp), _p(Vp), _p(None if pbf16 else ksc), _p(None if pbf16 else vsc), _p(row_state), _p(p_lo), _p(p_hi),
                                 _p(pmask), _p(Kq), _p(Vq), _p(row_q), _p(q_len), _p(k_own), _p(v_own), _p(own_lo),
                                 _p(own_hi), _p(row_groups),
                                 _p(out), _p(lse), dims, _p(ws), ws_bytes, _stream(dev)), "od_prefix_attn")
    return (out, lse) if want_lse else out


@_probed
def readout(logits: torch.Tensor, T: torch.Tensor, mask: torch.Tensor, bias: torch.Tensor | None = None,
            none_col: torch.Tensor | None = None, want_renorm: bool = True):
    """softmax(logits / T + bias) * mask -> probs (N, K) fp32; renorm (N, K) fp64; p_none (N,) fp32."""
    dev = _need_cuda(logits, T, mask, bias, none_col)
    N, K = logits.shape
    probs = torch.empty(N, K, dtype=torch.float32, device=dev)
    renorm = torch.empty(N, K, dtype=torch.float64, device=dev) if want_renorm else None
    p_none = torch.empty(N, dtype=torch.float32, device=dev) if none_col is not None else None
    _check(load().od_readout(_p(logits), _p(T), _p(bias), _p(mask), _p(none_col), N, K, _p(probs), _p(renorm),
                             _p(p_none), _stream(dev)), "od_readout")
    return probs, renorm, p_none


@_probed
def prefix_attn_noalloc(q: torch.Tensor, k_own: torch.Tensor, v_own: torch.Tensor, sm_scale: float, *, nsplit: int,
                        Kp=None, Vp=None, ksc=None, vsc=None, row_state=None, p_lo=None, p_hi=None, pmask=None,
                        Kq=None, Vq=None, row_q=None, q_len=None, own_lo=None, own_hi=None, row_groups=None,
                        max_group_rows: int = 1, out=None, want_lse: bool = False):
    """prefix_attn through od_prefix_attn_noalloc: the split workspace is the library's static device scratch (no
    allocation by the call; `out`/`lse` are the caller's). Calls on one device must be stream-ordered."""
    dev = _need_cuda(q, k_own, v_own, Kp, Kq)
    R, t, Hq, D = q.shape
    Hkv = k_own.shape[2]
    out = torch.empty_like(q) if out is None else out
    lse = torch.empty(R, Hq, t, dtype=torch.float32, device=dev) if want_lse else None
    S, T = (Kp.shape[0], Kp.shape[2]) if Kp is not None else (0, 0)
    NQ, Lq = (Kq.shape[0], Kq.shape[1]) if Kq is not None else (0, 0)
    pbf16 = Kp is not None and Kp.dtype == torch.bfloat16
    sdt = _DT[ksc.dtype] if (ksc is not None and not pbf16) else OD_BF16
    G = row_groups.shape[0] if row_groups is not None else R
    dims = AttnDims(R, t, S, T, NQ, Lq, Hq, Hkv, D, sdt, sm_scale, G, max_group_rows if row_groups is not None else 1,
                    1 if pbf16 else 0, nsplit)
    _check(load().od_prefix_attn_noalloc(
        _p(q), _p(Kp), _p(Vp), _p(None if pbf16 else ksc), _p(None if pbf16 else vsc), _p(row_state), _p(p_lo),
        _p(p_hi), _p(pmask), _p(Kq), _p(Vq), _p(row_q), _p(q_len), _p(k_own), _p(v_own), _p(own_lo), _p(own_hi),
        _p(row_groups), _p(out), _p(lse), dims, _stream(dev)), "od_prefix_attn_noalloc")
    return (out, lse) if want_lse else out


@_probed
def lm_logprob(h: torch.Tensor, Wb: torch.Tensor, qW: torch.Tensor, sW: torch.Tensor, tok: torch.Tensor,
               vsplit: int | None = None) -> torch.Tensor:
    """log softmax(h Wb^T)[tok] as Backbone.token_logprob computes it: h (M, H) bf16, Wb (V, H) bf16 (the dequantised
    tied head), qW (V, H) int8 + sW (V,) bf16 (the int8 head, for the fp32 target logit), tok (M,) int64 -> (M,)
    fp32. vsplit: vocabulary ranges per row tile (None: od_lm_logprob_plan's choice for this GPU)."""
    dev = _need_cuda(h, Wb, qW, sW, tok)
    M, H = h.shape
    V = Wb.shape[0]
    assert h.is_contiguous() and Wb.is_contiguous() and qW.is_contiguous() and tok.dtype == torch.int64
    assert Wb.shape == qW.shape == (V, H) and sW.numel() == V and h.dtype == Wb.dtype == torch.bfloat16
    n, b = ctypes.c_int(1), ctypes.c_int64(0)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    _check(load().od_lm_logprob_plan(M, V, sms, ctypes.byref(n), ctypes.byref(b)), "od_lm_logprob_plan")
    if vsplit is not None:
        n.value, b.value = vsplit, 8 * M * vsplit
    ws = torch.empty(max(1, b.value // 4), dtype=torch.float32, device=dev)
    lp = torch.empty(M, dtype=torch.float32, device=dev)
    _check(load().od_lm_logprob(_p(h), M, H, _p(Wb), _p(qW), _p(sW.contiguous()), V, _p(tok.contiguous()), _p(lp),
                                _p(ws), ws.numel() * 4, n.value, _stream(dev)), "od_lm_logprob")
    return lp


# ------------------------------------------------------------------------------------------------ V3 trunk (fp32)
# An fp32 GEMM operand travels as a pair (hi, lo) of (M, K) fp32 tensors with hi = x rounded to tf32 and lo = x - hi:
# od_gemm_f32 multiplies such pairs on the tensor cores (3 tf32 products per k-step) with fp32-level accuracy.


def _pair(M: int, K: int, dev) -> tuple:
    return (torch.empty(M, K, dtype=torch.float32, device=dev), torch.empty(M, K, dtype=torch.float32, device=dev))


@_probed
def split_tf32(x: torch.Tensor) -> tuple:
    """x (M, K) fp32 -> the operand pair (hi, lo) of gemm_f32."""
    dev = _need_cuda(x)
    assert x.dtype == torch.float32 and x.dim() == 2 and x.stride(1) == 1
    M, K = x.shape
    hi, lo = _pair(M, K, dev)
    _check(load().od_split_tf32(_p(x), x.stride(0), M, K, _p(hi), _p(lo), K, _stream(dev)), "od_split_tf32")
    return hi, lo


@_probed
def scalenorm_split(x: torch.Tensor, g: torch.Tensor, eps: float = 1e-5, mix_w: torch.Tensor | None = None) -> tuple:
    """ScaleNorm g * x / max(||x||, eps) per row (v3.py:43-50) as an operand pair; g a 0-dim fp32 device tensor.
    With mix_w (n,) fp32 the row is first sum_l mix_w[l] * x[:, l K:(l + 1) K] (the layer mix, v3.py:328-341).
    x (M, K) or (M, n K) in bf16 / fp16 / fp32, rows contiguous; a 1-D x is one row."""
    dev = _need_cuda(x, g, mix_w)
    x2 = x.view(1, -1) if x.dim() == 1 else x
    assert x2.stride(1) == 1 and g.dtype == torch.float32 and g.numel() == 1
    n = 1 if mix_w is None else mix_w.numel()
    M, K = x2.shape[0], x2.shape[1] // n
    hi, lo = _pair(M, K, dev)
    _check(load().od_scalenorm_split(_p(x2), _DT[x2.dtype], x2.stride(0), M, K, _p(mix_w), n, _p(g), eps, _p(hi),
                                     _p(lo), K, _stream(dev)), "od_scalenorm_split")
    return hi, lo


@_probed
def gemm_f32(x: tuple, w: tuple, bias: torch.Tensor | None = None, res: torch.Tensor | None = None,
             out: torch.Tensor | None = None, out_rows: torch.Tensor | None = None,
             rope_pos: torch.Tensor | None = None, rope_inv: torch.Tensor | None = None,
             rope_cols: int = 0) -> torch.Tensor:
    """y[out_rows[r]] = x[r] . W^T (+ bias) (+ res[out_rows[r]]) in fp32: x = (hi, lo) (M, K), w = (hi, lo) (N, K)
    (nn.Linear's layout), bias (N,), res (rows, N) - may be `out` itself (x = x + layer(x)) - or (N,) (one row for
    every output row), out_rows (M,) int64 (default: row r). rope_pos (M,) int32 with rope_inv (dh / 2,) fp32 (the
    frequencies, rope_table()): columns [0, rope_cols) leave RoPE'd in dh-wide heads (v3.py:70-79). Returns out
    ((M, N) fp32 when not given)."""
    xh, xl = x
    wh, wl = w
    dev = _need_cuda(xh, xl, wh, wl, bias, res, out, out_rows, rope_pos, rope_inv)
    M, K = xh.shape
    N = wh.shape[0]
    assert xl.shape == xh.shape and xl.stride(0) == xh.stride(0) and wl.shape == wh.shape
    assert wl.stride(0) == wh.stride(0) and wh.shape[1] == K and xh.stride(1) == 1 and wh.stride(1) == 1
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=dev)
    assert out.dtype == torch.float32 and out.stride(-1) == 1 and out.shape[-1] == N
    ldres = 0
    if res is not None:
        assert res.dtype == torch.float32 and res.stride(-1) == 1
        ldres = 0 if res.dim() == 1 else res.stride(0)
    if out_rows is not None:
        assert out_rows.dtype == torch.int64 and out_rows.numel() == M
    rope_dh = 0
    if rope_pos is not None:
        assert rope_pos.dtype == torch.int32 and rope_pos.is_contiguous() and rope_pos.numel() == M
        assert rope_inv is not None and rope_inv.dtype == torch.float32 and rope_inv.is_contiguous()
        rope_dh = 2 * rope_inv.numel()
    _check(load().od_gemm_f32(_p(xh), _p(xl), xh.stride(0), _p(wh), _p(wl), wh.stride(0), _p(bias), _p(res), ldres,
                              _p(out_rows), _p(rope_pos), _p(rope_inv), rope_cols, rope_dh, _p(out), out.stride(0),
                              M, N, K, _stream(dev)), "od_gemm_f32")
    return out


def rope_table(dh: int, device) -> torch.Tensor:
    """The trunk RoPE's frequencies 1 / 10000^(2i / dh), i < dh / 2, evaluated in fp32 by torch on the host exactly
    as the reference's rope() writes them (v3.py:75), for gemm_f32's RoPE epilogue."""
    inv = 1.0 / (10000 ** (torch.arange(0, dh, 2, dtype=torch.float32) / dh))
    return inv.to(device)


@_probed
def xatglu_split(zv: torch.Tensor, alpha: torch.Tensor) -> tuple:
    """zv (M, 2F) = [wg x + bg | wv x + bv] -> the XATGLU product (((atan z + pi/2) / pi)(1 + 2a) - a) * value
    (v3.py:65-66) as an operand pair (M, F); alpha a 0-dim fp32 device tensor."""
    dev = _need_cuda(zv, alpha)
    assert zv.dtype == torch.float32 and zv.stride(1) == 1 and zv.shape[1] % 2 == 0
    M, F = zv.shape[0], zv.shape[1] // 2
    hi, lo = _pair(M, F, dev)
    _check(load().od_xatglu_split(_p(zv), zv.stride(0), M, F, _p(alpha), _p(hi), _p(lo), F, _stream(dev)),
           "od_xatglu_split")
    return hi, lo


@_probed
def trunk_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mode: int, B: int, Lq: int, Lk: int, H: int,
               k_grp: torch.Tensor, q_grp: torch.Tensor | None = None, bonus: torch.Tensor | None = None,
               q_shared: bool = False, q_len: torch.Tensor | None = None, k_len: torch.Tensor | None = None,
               pair: bool = True):
    """One trunk MHA's attention (v3.py:97) with its mask from ids (od_trunk_attn): q (B * Lq, H * Dh) rows (or one
    row shared by every query when q_shared), k / v (B * Lk, H * Dh) rows (column slices of a wider buffer allowed),
    q and k already RoPE'd, groups (B, L) int32, q_len / k_len (B,) int32 the real (prefix) lengths or None. Returns
    the output (B * Lq, H * Dh) as an operand pair (pair=True) or fp32; padding queries get zeros."""
    dev = _need_cuda(q, k, v, k_grp, q_grp, bonus, q_len, k_len)
    D = q.shape[-1]
    Dh = D // H
    assert q.stride(-1) == 1 and k.stride(-1) == 1 and v.stride(-1) == 1 and k.stride(0) == v.stride(0)
    for t in (k_grp, q_grp, q_len, k_len):
        assert t is None or (t.dtype == torch.int32 and t.is_contiguous())
    ldq = 0 if q_shared else q.stride(0)
    qbs = 0 if q_shared else Lq * q.stride(0)
    if pair:
        o = None
        hi, lo = _pair(B * Lq, D, dev)
    else:
        o = torch.empty(B * Lq, D, dtype=torch.float32, device=dev)
        hi = lo = None
    _check(load().od_trunk_attn(_p(q), ldq, qbs, _p(k), _p(v), k.stride(0), Lk * k.stride(0), _p(q_grp),
                                _p(k_grp), _p(bonus), _p(q_len), _p(k_len), mode, B, Lq, Lk, H, Dh, _p(o), _p(hi),
                                _p(lo), D,
                                _stream(dev)), "od_trunk_attn")
    return (hi, lo) if pair else o


def selftest_bounded_wait(limit_cycles: int, device=None) -> None:
    """Launch the failure-detection self-test (od_selftest_bounded_wait): a wait that runs out after limit_cycles and
    records its code in the device error word (read it with device_error())."""
    dev = torch.device(device or "cuda")
    _check(load().od_selftest_bounded_wait(int(limit_cycles), _stream(dev)), "od_selftest_bounded_wait")
