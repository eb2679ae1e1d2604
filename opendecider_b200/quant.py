"""int8 tensors and W8A8 linears on libod_b200 - the reference's quant.py seams (src/opendecider/quant.py) on B200.

Same layouts and the same quantiser as the reference:
  Int8Tensor      q int8 + one scale per row over the last dim, scale in the source dtype (quant.py:30-58)
  Int8Linear      qweight (N, K) int8 + scale (N, 1) in the weight dtype (quant.py:119-164); forward() calls the
                  `_fused` slot when one is installed (quant.py:149-152), the seam the W8A8 kernel plugs into
  W8A8            the fused callable for that slot: per-token int8 activations (od_quant_rows_i8, optionally with
                  SmoothQuant's inv_s multiply fused, quant.py:317-329) + the tcgen05 int8 GEMM (od_gemm_w8a8) with
                  the dequant epilogue. Replaces GemLite's A8W8 (quant.py:302-314) and the dequant + cuBLAS path.
Everything runs on CUDA tensors; there is no CPU path (a CPU tensor raises ODError).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib


@dataclass
class Int8Tensor:
    q: torch.Tensor          # int8, same shape as the original
    scale: torch.Tensor      # shape[:-1] (+ (1,) in the reference), original dtype
    dtype: torch.dtype

    @classmethod
    def quantize(cls, x: torch.Tensor) -> "Int8Tensor":
        """Int8Tensor.quantize (quant.py:37-41) on the GPU: bit-identical bytes and scales."""
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) != x2.shape[1]):
            x2 = x2.contiguous()
        sdt = x.dtype if x.dtype != torch.float32 else torch.float32
        q, s = _lib.quant_rows(x2, scale_dtype=sdt)
        return cls(q.view(x.shape), s.view(*x.shape[:-1], 1), x.dtype)

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        dt = dtype or self.dtype
        y = _lib.dequant_rows(self.q.reshape(-1, self.q.shape[-1]), self.scale.reshape(-1, 1), dt)
        return y.view(self.q.shape)

    @property
    def shape(self):
        return self.q.shape

    def nbytes(self) -> int:
        return self.q.numel() + self.scale.numel() * self.scale.element_size()

    def index_select(self, dim: int, idx: torch.Tensor) -> "Int8Tensor":
        return Int8Tensor(self.q.index_select(dim, idx), self.scale.index_select(dim, idx), self.dtype)


def quantize_weight(w: torch.Tensor):
    """Int8Linear.__init__'s quantiser (quant.py:124-127) on the device: (qweight (N, K) int8, scale (N, 1))."""
    assert w.is_cuda, "weights are quantised on the GPU (no CPU path)"
    return _lib.quant_rows(w.contiguous(), scale_dtype=w.dtype if w.dtype != torch.float32 else torch.float32)


class W8A8(nn.Module):
    """The `_fused` callable of one Int8Linear: fused(x (..., K) bf16) -> (..., N) bf16 through od_quant_rows_i8 +
    od_gemm_w8a8. Holds the SAME int8 bytes as the Int8Linear (its qweight/scale tensors, no copy). inv_s: the
    SmoothedLinear per-channel multiply, fused into the activation quantiser. K % 128 == 0 and N % 256 == 0."""

    def __init__(self, qweight: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None,
                 inv_s: torch.Tensor | None = None):
        super().__init__()
        self.qweight, self.scale = qweight, scale.reshape(-1).to(torch.bfloat16).contiguous()
        self.bias, self.inv_s = bias, inv_s
        self.out_features, self.in_features = qweight.shape

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if x2.dtype != torch.bfloat16:
            raise _lib.ODError("W8A8 takes bf16 activations")
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        xq, sx = _lib.quant_rows(x2, scale_dtype=torch.float32, inv_s=self.inv_s)
        y = _lib.gemm_w8a8(xq, sx.view(-1), self.qweight, self.scale, _lib.OD_EPI_BF16)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        return y.view(*shp[:-1], self.out_features)

    def dense_weight(self) -> torch.Tensor:
        """(in, out) dequantised weight, for code paths that read `.weight` (Int8Linear.weight, quant.py:134-140)."""
        return (self.qweight.to(self.scale.dtype) * self.scale[:, None]).t()


class Int8Linear(nn.Module):
    """Frozen int8 linear in the reference's layout (quant.py:119-164). forward() dispatches to the `_fused` slot;
    without one it runs the W8A8 kernel on its own buffers (there is no dequantise + dense fallback)."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        w = lin.weight.data
        q, s = quantize_weight(w)
        self.register_buffer("qweight", q)
        self.register_buffer("scale", s)
        self.bias = None if lin.bias is None else lin.bias.data.clone()
        self.in_features, self.out_features = lin.in_features, lin.out_features

    @property
    def weight(self) -> torch.Tensor:
        f = self.__dict__.get("_fused")
        if f is not None:
            return f.dense_weight().t()
        return self.qweight.to(self.scale.dtype) * self.scale

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        fused = self.__dict__.get("_fused")
        if fused is None:
            fused = W8A8(self.qweight, self.scale, self.bias)
            self.__dict__["_fused"] = fused
        return fused(x)


def b200_int8_kernels_(module: nn.Module, smooth: dict | None = None) -> int:
    """Give every Int8Linear under `module` (the reference's class or this one: anything with int8 `qweight` and a
    `scale`) a W8A8 `_fused` kernel on the SAME weights - the seam int8_to_gemlite_ fills (quant.py:398-409). The
    module objects stay in place, so forward hooks on them keep working. smooth: {module name: inv_s bf16 (K,)}.
    Returns the number of layers given a kernel."""
    n = 0
    for name, m in module.named_modules():
        q = getattr(m, "qweight", None)
        if isinstance(q, torch.Tensor) and q.dtype == torch.int8 and q.numel() and hasattr(m, "scale") \
                and m.__dict__.get("_dq") is None:
            inv = None if smooth is None else smooth.get(name)
            m.__dict__["_fused"] = W8A8(q, m.scale, getattr(m, "bias", None), inv)
            n += 1
    return n
