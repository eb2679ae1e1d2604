// Bandwidth-bound row kernels of the decision forward pass: per-row int8 quantisation (weights, activations, KV),
// dequantisation, the int8 KV-cache append, fused residual + RMSNorm + quantisation, the int8 embedding lookup,
// the attention output gate + quantisation, and the option readout softmax.
//
// Every kernel reads its input once from HBM and keeps the row in registers between the reduction and the write,
// with 16-byte vector accesses that are coalesced across the threads of a row block. Rounding follows the
// reference's PyTorch ops one op at a time (see the comments at each step).
#include "common.cuh"

namespace od {
namespace {

constexpr int kRowThreads = 256;  // one CTA per row; a row of K elements is K / 8 vectors of 8

// ---------------------------------------------------------------------------------------------- vector I/O
template <typename T> __device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <> __device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
  uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T> __device__ __forceinline__ void store8(T* p, const float (&v)[8]);
template <> __device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ void store8_i8(int8_t* p, const float (&v)[8], float s, float r) {
  *reinterpret_cast<uint2*>(p) = quant8(v, s, r);
}

// Round a value to the precision of T (the dtype a PyTorch op on T tensors stores).
template <typename T> __device__ __forceinline__ float round_to(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

// Block-wide reductions over kRowThreads threads.
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kRowThreads / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < kRowThreads / 32; ++i) r += red[i];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------------------------- quantise rows
// Int8Tensor.quantize (quant.py:37-41) per row; optional SmoothedLinear multiply first (quant.py:328-329).
template <typename T, int VPT>
__global__ void __launch_bounds__(kRowThreads) quant_rows_kernel(const T* __restrict__ x, int64_t K, int64_t ldx,
                                                                 const __nv_bfloat16* __restrict__ inv_s,
                                                                 int8_t* __restrict__ q, void* scale,
                                                                 int scale_dtype) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  float v[VPT][8];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    if (e < K) {
      load8<T>(xr + e, v[j]);
      if (inv_s) {
        float w[8];
        load8<__nv_bfloat16>(inv_s + e, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = round_to<T>(v[j][i] * round_to<T>(w[i]));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[j][i]));
    }
  }
  amax = block_max(amax, red);
  const float s = quant_scale(amax), rs = quant_recip(s);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    if (e < K) store8_i8(q + row * K + e, v[j], s, rs);
  }
  if (threadIdx.x == 0) store_scale(scale, row, s, scale_dtype);
}

// The bf16 form without SmoothQuant (the activation path): the row stays packed, absmax by bf16 pair max.
template <int VPT>
__global__ void __launch_bounds__(kRowThreads) quant_rows_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t K,
                                                                      int64_t ldx, int8_t* __restrict__ q, void* scale,
                                                                      int scale_dtype) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  uint4 v[VPT];
  uint32_t am = 0u;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    v[j] = e < K ? __ldg(reinterpret_cast<const uint4*>(xr + e)) : make_uint4(0, 0, 0, 0);
    am = babsmax4(v[j], am);
  }
  const float amax = block_max(bmax_halves(am), red);
  const float s = quant_scale(amax), rs = quant_recip(s);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    if (e < K) {
      float f[8];
      unpack8(v[j], f);
      *reinterpret_cast<uint2*>(q + row * K + e) = quant8(f, s, rs);
    }
  }
  if (threadIdx.x == 0) store_scale(scale, row, s, scale_dtype);
}

template <typename T>
int launch_quant_rows(const T* x, int64_t M, int64_t K, int64_t ldx, const __nv_bfloat16* inv_s, int8_t* q,
                      void* scale, int scale_dtype, cudaStream_t st) {
  const int64_t vecs = (K / 8 + kRowThreads - 1) / kRowThreads;
  dim3 grid(static_cast<unsigned>(M)), block(kRowThreads);
  if (std::is_same<T, __nv_bfloat16>::value && !inv_s && vecs <= 16 && ldx % 8 == 0) {
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
#define OD_QB(V) quant_rows_bf16_kernel<V><<<grid, block, 0, st>>>(xb, K, ldx, q, scale, scale_dtype)
    if (vecs <= 1) OD_QB(1);
    else if (vecs <= 2) OD_QB(2);
    else if (vecs <= 3) OD_QB(3);
    else if (vecs <= 4) OD_QB(4);
    else if (vecs <= 6) OD_QB(6);
    else if (vecs <= 8) OD_QB(8);
    else if (vecs <= 12) OD_QB(12);
    else OD_QB(16);
#undef OD_QB
    OD_LAUNCH_CHECK();
    return ok();
  }
#define OD_QR(V) quant_rows_kernel<T, V><<<grid, block, 0, st>>>(x, K, ldx, inv_s, q, scale, scale_dtype)
  if (vecs <= 1) OD_QR(1);
  else if (vecs <= 2) OD_QR(2);
  else if (vecs <= 3) OD_QR(3);
  else if (vecs <= 4) OD_QR(4);
  else if (vecs <= 6) OD_QR(6);
  else if (vecs <= 8) OD_QR(8);
  else if (vecs <= 12) OD_QR(12);
  else if (vecs <= 16) OD_QR(16);
  else return fail(OD_EUNSUPPORTED, "od_quant_rows_i8: K=%lld above %d", (long long)K, 16 * 8 * kRowThreads);
#undef OD_QR
  OD_LAUNCH_CHECK();
  return ok();
}

// ---------------------------------------------------------------------------------------------- dequantise rows
template <typename TO>
__global__ void dequant_rows_kernel(const int8_t* __restrict__ q, const void* scale, int scale_dtype, int64_t M,
                                    int64_t K, TO* __restrict__ y) {
  const int64_t n = M * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K;
    // Int8Tensor.dequantize: q.to(dt) * scale.to(dt), one rounding of the product to dt
    const float s = round_to<TO>(load_scale(scale, r, scale_dtype));
    y[i] = Elem<TO>::from_f(static_cast<float>(q[i]) * s);
  }
}

// bf16 output with bf16 scales and rows of a multiple of 16: one 16-byte int8 chunk per thread and step, the exact
// integer-path conversion (RN(q * s) in bf16, as the scalar kernel rounds); 32-bit chunk indices.
__global__ void dequant_rows_bf16_kernel(const int8_t* __restrict__ q, const uint16_t* __restrict__ scale, uint32_t K16,
                                         uint32_t n, __nv_bfloat16* __restrict__ y) {
  for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    const uint32_t sb = __ldg(scale + c / K16);
    const uint32_t s2 = sb | (sb << 16);
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(q) + c);
    uint32_t o[8];
    dequant4_bf16(w.x, s2, o[0], o[1]);
    dequant4_bf16(w.y, s2, o[2], o[3]);
    dequant4_bf16(w.z, s2, o[4], o[5]);
    dequant4_bf16(w.w, s2, o[6], o[7]);
    uint4* dst = reinterpret_cast<uint4*>(y) + 2 * static_cast<uint64_t>(c);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
}

// ---------------------------------------------------------------------------------------------- KV append
// One warp per (state, new token, head) row of D elements; EPL = D / 32 contiguous elements per lane. The grid's y
// index is the state, x covers the (token, head) rows of one state (32-bit index arithmetic).
template <typename T, int EPL>
__global__ void kv_append_kernel(const T* __restrict__ k, const T* __restrict__ v, int64_t S, int64_t t, int Hkv,
                                 int64_t ks_s, int64_t ks_t, int64_t ks_h, int64_t vs_s, int64_t vs_t, int64_t vs_h,
                                 int8_t* __restrict__ kq, int8_t* __restrict__ vq, T* __restrict__ ksc,
                                 T* __restrict__ vsc, T* __restrict__ kb, T* __restrict__ vb, int64_t T_cap,
                                 int64_t t0, bool vec) {
  constexpr int D = EPL * 32;
  const int item = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= static_cast<int>(t) * Hkv) return;
  const int64_t j = item / Hkv;
  const int h = item - static_cast<int>(j) * Hkv;
  const int64_t s = blockIdx.y;
  const int64_t dst = ((s * Hkv + h) * T_cap + t0 + j);
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const T* src = (which == 0 ? k + s * ks_s + j * ks_t + h * ks_h : v + s * vs_s + j * vs_t + h * vs_h) + lane * EPL;
    float x[EPL];
    if (EPL == 4 && sizeof(T) == 2 && vec) {             // one 8-byte load per lane
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(src));
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = Elem<T>::to_f(e[i]);
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) x[i] = Elem<T>::to_f(src[i]);
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(x[i]));
    amax = warp_max(amax);
    const float sc = quant_scale(amax), rs = quant_recip(sc);
    int8_t* out = (which == 0 ? kq : vq) + dst * D + lane * EPL;
    int8_t qv[EPL];
    if (EPL == 4 && vec) {                                // one 4-byte store per lane
      const uint32_t w = quant4(x[0], x[1], x[2], x[3], sc, rs);
      *reinterpret_cast<uint32_t*>(out) = w;
#pragma unroll
      for (int i = 0; i < EPL; ++i) qv[i] = static_cast<int8_t>(w >> (8 * i));
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        qv[i] = quant_val(x[i], sc, rs);
        out[i] = qv[i];
      }
    }
    const T sc_t = Elem<T>::from_f(sc);
    if (lane == 0) (which == 0 ? ksc : vsc)[dst] = sc_t;
    T* mat = which == 0 ? kb : vb;
    if (mat != nullptr) {   // materialize(): q * s in the scale's dtype; |q| <= 127 times s is exact in fp32
      const float sf = Elem<T>::to_f(sc_t);
      T m[EPL];
#pragma unroll
      for (int i = 0; i < EPL; ++i) m[i] = Elem<T>::from_f(static_cast<float>(qv[i]) * sf);
      T* mo = mat + dst * D + lane * EPL;
      if constexpr (EPL * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(mo) = *reinterpret_cast<const uint4*>(m);
      } else if constexpr (EPL * sizeof(T) == 8) {
        *reinterpret_cast<uint2*>(mo) = *reinterpret_cast<const uint2*>(m);
      } else if constexpr (EPL * sizeof(T) == 4) {
        *reinterpret_cast<uint32_t*>(mo) = *reinterpret_cast<const uint32_t*>(m);
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i) mo[i] = m[i];
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------- norm + quant
// Residual add + Qwen3_5RMSNorm + optional SmoothQuant multiply + per-token quantisation, one row per CTA.
template <int VPT>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_res_quant_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res_in, __nv_bfloat16* res_out,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ inv_s, float eps, int H,
    __nv_bfloat16* __restrict__ y_out, int8_t* __restrict__ q, float* __restrict__ s_out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int64_t base = row * H;
  uint4 hv[VPT];                                      // the row (hidden, then y), packed bf16
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = (j * kRowThreads + threadIdx.x) * 8;
    hv[j] = make_uint4(0, 0, 0, 0);
    if (e < H) {
      uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + base + e));
      if (res_in) {  // hidden = residual + hidden, one bf16 rounding
        const uint4 rv = __ldg(reinterpret_cast<const uint4*>(res_in + base + e));
        xv = make_uint4(badd2(rv.x, xv.x), badd2(rv.y, xv.y), badd2(rv.z, xv.z), badd2(rv.w, xv.w));
        *reinterpret_cast<uint4*>(res_out + base + e) = xv;
      }
      hv[j] = xv;
      float f[8];
      unpack8(xv, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
  }
  ss = block_sum(ss, red);
  // torch.rsqrt(x.pow(2).mean(-1) + eps): mean in fp32, then 1 / sqrt (the CPU reference rounds twice)
  const float var = __fdiv_rn(ss, static_cast<float>(H));
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const float2 rs2 = make_float2(rs, rs), one2 = make_float2(1.0f, 1.0f);
  uint32_t am = 0u;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = (j * kRowThreads + threadIdx.x) * 8;
    if (e < H) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + e));
      const uint32_t* hw = &hv[j].x;
      const uint32_t* ww = &wv.x;
      uint32_t y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {               // y = bf16((h * rs) * (1 + w))
        const float2 v = __fmul2_rn(__fmul2_rn(unpack2(hw[i]), rs2), __fadd2_rn(one2, unpack2(ww[i])));
        y[i] = pack_rn(v.x, v.y);
      }
      if (inv_s) {                                 // SmoothQuant: bf16(y * inv_s)
        const uint4 is = __ldg(reinterpret_cast<const uint4*>(inv_s + e));
        y[0] = bmul2(y[0], is.x);
        y[1] = bmul2(y[1], is.y);
        y[2] = bmul2(y[2], is.z);
        y[3] = bmul2(y[3], is.w);
      }
      hv[j] = make_uint4(y[0], y[1], y[2], y[3]);
      if (y_out) *reinterpret_cast<uint4*>(y_out + base + e) = hv[j];
      am = babsmax4(hv[j], am);
    }
  }
  if (!q) return;
  const float amax = block_max(bmax_halves(am), red);
  const float sc = quant_scale(amax), rq = quant_recip(sc);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = (j * kRowThreads + threadIdx.x) * 8;
    if (e < H) {
      float f[8];
      unpack8(hv[j], f);
      *reinterpret_cast<uint2*>(q + base + e) = quant8(f, sc, rq);
    }
  }
  if (threadIdx.x == 0) s_out[row] = sc;
}

// ---------------------------------------------------------------------------------------------- embedding
__global__ void embed_i8_kernel(const int64_t* __restrict__ ids, const int8_t* __restrict__ qw,
                                const __nv_bfloat16* __restrict__ scale, int64_t V, int H,
                                __nv_bfloat16* __restrict__ out, int32_t* err) {
  const int64_t tok = blockIdx.x;
  int64_t id = ids[tok];
  if (id < 0 || id >= V) {  // out-of-range id: record it and write zeros instead of reading out of bounds
    if (threadIdx.x == 0) atomicCAS(err, 0, 0x1D0000 | 1);
    id = -1;
  }
  const float s = id >= 0 ? __bfloat162float(scale[id]) : 0.f;
  for (int e = threadIdx.x * 8; e < H; e += blockDim.x * 8) {
    float v[8];
    if (id >= 0) {
      uint2 raw = *reinterpret_cast<const uint2*>(qw + id * H + e);
      const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = rbf(static_cast<float>(b[i]) * s);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    store8<__nv_bfloat16>(out + tok * H + e, v);
  }
}

// ---------------------------------------------------------------------------------------------- gate + quant
// sigmoid(g) = 1 / (1 + exp(-g)) in fp32 (expf, IEEE division), rounded to bf16. A fast value from the hardware
// exp2 / reciprocal approximations (relative error below 1.4e-6 for |g| < 16) rounds to the same bf16 unless a bf16
// rounding boundary - a tie, low 16 bits 0x8000 - lies between the two: so only a fast value within 64 fp32 ulps
// (relative 3.8e-6) of a tie, or |g| >= 16, takes the fp32 formula. (Crossing a bf16-representable value changes
// the upper bits but both sides round to that value.)
// Two sigmoids packed as a bf16 pair (lo = g.x), the pair's arithmetic in packed fp32 operations. A value is near a
// tie when its low 16 bits lie within 64 of 0x8000: (bits + 0x803F) mod 2^16 below 0x80.
__device__ __forceinline__ uint32_t sigmoid2_bf16(float2 g) {
  const float2 y = __fmul2_rn(g, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  float e0, e1, v0, v1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(y.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(y.y));
  const float2 d = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(e0, e1));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(v0) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(v1) : "f"(d.y));
  const uint32_t t0 = (__float_as_uint(v0) + 0x803Fu) & 0xFF80u, t1 = (__float_as_uint(v1) + 0x803Fu) & 0xFF80u;
  if (min(t0, t1) == 0u || fmaxf(fabsf(g.x), fabsf(g.y)) >= 16.0f) {
    v0 = __fdiv_rn(1.0f, 1.0f + expf(-g.x));
    v1 = __fdiv_rn(1.0f, 1.0f + expf(-g.y));
  }
  return pack_rn(v0, v1);
}

// o * sigmoid(gate) (Qwen3_5Attention.forward), the o_proj SmoothedLinear multiply when inv_s is given, then
// per-token quantisation of the o_proj input.
template <int VPT>
__global__ void __launch_bounds__(kRowThreads) gate_quant_kernel(const __nv_bfloat16* __restrict__ o,
                                                                 const __nv_bfloat16* __restrict__ qkv,
                                                                 int64_t ldqkv, int Hq, int D,
                                                                 const __nv_bfloat16* __restrict__ inv_s,
                                                                 int8_t* __restrict__ q, float* __restrict__ s_out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const int W = Hq * D;
  uint4 vv[VPT];                                      // bf16(o * sigmoid(gate)), packed
  uint32_t am = 0u;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = (j * kRowThreads + threadIdx.x) * 8;
    vv[j] = make_uint4(0, 0, 0, 0);
    if (e < W) {
      const int h = e / D, d = e - h * D;
      const uint4 ov = __ldg(reinterpret_cast<const uint4*>(o + row * W + e));
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(qkv + row * ldqkv + static_cast<int64_t>(h) * 2 * D + D + d));
      vv[j] = make_uint4(bmul2(ov.x, sigmoid2_bf16(unpack2(gv.x))), bmul2(ov.y, sigmoid2_bf16(unpack2(gv.y))),
                         bmul2(ov.z, sigmoid2_bf16(unpack2(gv.z))), bmul2(ov.w, sigmoid2_bf16(unpack2(gv.w))));
      if (inv_s) {                                   // SmoothedLinear: bf16(x * inv_s)
        const uint4 is = __ldg(reinterpret_cast<const uint4*>(inv_s + e));
        vv[j] = make_uint4(bmul2(vv[j].x, is.x), bmul2(vv[j].y, is.y), bmul2(vv[j].z, is.z), bmul2(vv[j].w, is.w));
      }
      am = babsmax4(vv[j], am);
    }
  }
  const float amax = block_max(bmax_halves(am), red);
  const float sc = quant_scale(amax), rq = quant_recip(sc);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = (j * kRowThreads + threadIdx.x) * 8;
    if (e < W) {
      float f[8];
      unpack8(vv[j], f);
      *reinterpret_cast<uint2*>(q + row * W + e) = quant8(f, sc, rq);
    }
  }
  if (threadIdx.x == 0) s_out[row] = sc;
}

// SwiGLU of separately computed gate and up projections (Qwen3_5MLP.forward: act_fn(gate_proj(x)) * up_proj(x)),
// with the rounding points of the GEMM's fused SwiGLU epilogue: a = bf16(g / (1 + exp(-g))), h = bf16(a * u); then
// the down projection's SmoothedLinear multiply when inv_s is given and per-token quantisation (its input). Used
// when gate_proj and up_proj are smoothed by different vectors and so cannot share one interleaved GEMM.
template <int VPT>
__global__ void __launch_bounds__(kRowThreads) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ g,
                                                                   const __nv_bfloat16* __restrict__ u, int64_t F,
                                                                   const __nv_bfloat16* __restrict__ inv_s,
                                                                   int8_t* __restrict__ q, float* __restrict__ s_out) {
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  uint4 hv[VPT];
  uint32_t am = 0u;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    hv[j] = make_uint4(0, 0, 0, 0);
    if (e < F) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(g + row * F + e));
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(u + row * F + e));
      float gf[8];
      unpack8(gv, gf);
      uint32_t a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = pack_rn(__fdiv_rn(gf[2 * i], 1.0f + expf(-gf[2 * i])),
                       __fdiv_rn(gf[2 * i + 1], 1.0f + expf(-gf[2 * i + 1])));
      hv[j] = make_uint4(bmul2(a[0], uv.x), bmul2(a[1], uv.y), bmul2(a[2], uv.z), bmul2(a[3], uv.w));
      if (inv_s) {
        const uint4 is = __ldg(reinterpret_cast<const uint4*>(inv_s + e));
        hv[j] = make_uint4(bmul2(hv[j].x, is.x), bmul2(hv[j].y, is.y), bmul2(hv[j].z, is.z), bmul2(hv[j].w, is.w));
      }
      am = babsmax4(hv[j], am);
    }
  }
  const float amax = block_max(bmax_halves(am), red);
  const float sc = quant_scale(amax), rq = quant_recip(sc);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t e = (static_cast<int64_t>(j) * kRowThreads + threadIdx.x) * 8;
    if (e < F) {
      float f[8];
      unpack8(hv[j], f);
      *reinterpret_cast<uint2*>(q + row * F + e) = quant8(f, sc, rq);
    }
  }
  if (threadIdx.x == 0) s_out[row] = sc;
}

// ---------------------------------------------------------------------------------------------- readout
// Decider._probs softmax (decider.py:255-257) and _normalize (:26-29), one warp per question.
__global__ void readout_kernel(const float* __restrict__ logits, const float* __restrict__ T,
                               const float* __restrict__ bias, const uint8_t* __restrict__ mask,
                               const int32_t* __restrict__ none_col, int64_t N, int64_t K, float* __restrict__ probs,
                               double* __restrict__ renorm, float* __restrict__ p_none) {
  const int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= N) return;
  const float ti = T[i];
  float m = -INFINITY;
  for (int64_t k = lane; k < K; k += 32) {
    float z = __fdiv_rn(logits[i * K + k], ti);
    if (bias) z = __fadd_rn(z, bias[i * K + k]);
    m = fmaxf(m, z);
  }
  m = warp_max(m);
  float sum = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    float z = __fdiv_rn(logits[i * K + k], ti);
    if (bias) z = __fadd_rn(z, bias[i * K + k]);
    sum += expf(z - m);
  }
  sum = warp_sum(sum);
  const int nc = none_col ? none_col[i] : -1;
  const int64_t Kc = nc >= 0 ? nc : K;
  double dsum = 0.0;
  for (int64_t k = lane; k < K; k += 32) {
    float z = __fdiv_rn(logits[i * K + k], ti);
    if (bias) z = __fadd_rn(z, bias[i * K + k]);
    const float p = __fdiv_rn(expf(z - m), sum) * static_cast<float>(mask[i * K + k] != 0);
    probs[i * K + k] = p;
    if (k < Kc) dsum += fmax(static_cast<double>(p), 0.0);
    if (p_none && k == nc) p_none[i] = p;
  }
  if (p_none && nc < 0 && lane == 0) p_none[i] = 0.f;
  if (!renorm) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  for (int64_t k = lane; k < K; k += 32) {
    const double p = fmax(static_cast<double>(probs[i * K + k]), 0.0);
    renorm[i * K + k] = k < Kc ? p / dsum : 0.0;
  }
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_quant_rows_i8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const void* inv_s,
                                int8_t* q, void* scale, int scale_dtype, void* stream) {
  OD_REQUIRE(x && q && scale, "od_quant_rows_i8: null pointer");
  OD_REQUIRE(M >= 0 && K > 0 && K % 8 == 0 && ldx >= K && ldx % 8 == 0, "od_quant_rows_i8: bad shape M=%lld K=%lld ldx=%lld",
             (long long)M, (long long)K, (long long)ldx);
  OD_REQUIRE(aligned16(x) && aligned16(q) && (!inv_s || aligned16(inv_s)), "od_quant_rows_i8: pointers must be 16-byte aligned");
  OD_REQUIRE(scale_dtype >= OD_BF16 && scale_dtype <= OD_F32, "od_quant_rows_i8: bad scale dtype");
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const __nv_bfloat16* is = static_cast<const __nv_bfloat16*>(inv_s);
  switch (x_dtype) {
    case OD_BF16: return launch_quant_rows(static_cast<const __nv_bfloat16*>(x), M, K, ldx, is, q, scale, scale_dtype, st);
    case OD_F16: return launch_quant_rows(static_cast<const __half*>(x), M, K, ldx, is, q, scale, scale_dtype, st);
    case OD_F32: return launch_quant_rows(static_cast<const float*>(x), M, K, ldx, is, q, scale, scale_dtype, st);
    default: return fail(OD_EINVAL, "od_quant_rows_i8: bad x dtype %d", x_dtype);
  }
}

extern "C" int od_dequant_rows_i8(const int8_t* q, const void* scale, int scale_dtype, int64_t M, int64_t K, void* y,
                                  int out_dtype, void* stream) {
  OD_REQUIRE(q && scale && y, "od_dequant_rows_i8: null pointer");
  OD_REQUIRE(M >= 0 && K > 0, "od_dequant_rows_i8: bad shape");
  OD_REQUIRE(scale_dtype >= OD_BF16 && scale_dtype <= OD_F32, "od_dequant_rows_i8: bad scale dtype");
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const int64_t n = M * K;
  if (out_dtype == OD_BF16 && scale_dtype == OD_BF16 && K % 16 == 0 && n / 16 < (1LL << 32) - 65536 && aligned16(q) &&
      aligned16(y)) {
    const int64_t n16 = n / 16;
    const unsigned blocks = static_cast<unsigned>(n16 / 256 + 1 < 148 * 16 ? n16 / 256 + 1 : 148 * 16);
    dequant_rows_bf16_kernel<<<blocks, 256, 0, st>>>(q, static_cast<const uint16_t*>(scale),
                                                     static_cast<uint32_t>(K / 16), static_cast<uint32_t>(n16),
                                                     static_cast<__nv_bfloat16*>(y));
    OD_LAUNCH_CHECK();
    return ok();
  }
  const int blocks = static_cast<int>(n / 256 + 1 < 148 * 32 ? n / 256 + 1 : 148 * 32);
  switch (out_dtype) {
    case OD_BF16: dequant_rows_kernel<<<blocks, 256, 0, st>>>(q, scale, scale_dtype, M, K, static_cast<__nv_bfloat16*>(y)); break;
    case OD_F16: dequant_rows_kernel<<<blocks, 256, 0, st>>>(q, scale, scale_dtype, M, K, static_cast<__half*>(y)); break;
    case OD_F32: dequant_rows_kernel<<<blocks, 256, 0, st>>>(q, scale, scale_dtype, M, K, static_cast<float*>(y)); break;
    default: return fail(OD_EINVAL, "od_dequant_rows_i8: bad out dtype %d", out_dtype);
  }
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_kv_append_i8(const void* k, const void* v, int kv_dtype, int64_t S, int64_t t, int Hkv, int D,
                               int64_t ks_s, int64_t ks_t, int64_t ks_h, int64_t vs_s, int64_t vs_t, int64_t vs_h,
                               int8_t* kq, int8_t* vq, void* ksc, void* vsc, void* kb, void* vb, int64_t T_cap,
                               int64_t t0, void* stream) {
  OD_REQUIRE(k && v && kq && vq && ksc && vsc, "od_kv_append_i8: null pointer");
  OD_REQUIRE((kb == nullptr) == (vb == nullptr), "od_kv_append_i8: kb and vb go together");
  OD_REQUIRE(kb == nullptr || ((reinterpret_cast<uintptr_t>(kb) | reinterpret_cast<uintptr_t>(vb)) & 15) == 0,
             "od_kv_append_i8: materialised outputs must be 16-byte aligned");
  OD_REQUIRE(S >= 0 && t >= 0 && Hkv > 0 && t0 >= 0 && t0 + t <= T_cap, "od_kv_append_i8: bad shape (t0 + t > T_cap?)");
  OD_REQUIRE(D == 64 || D == 128 || D == 256, "od_kv_append_i8: head_dim %d not in {64, 128, 256}", D);
  if (S == 0 || t == 0) return ok();
  cudaStream_t st = as_stream(stream);
  OD_REQUIRE(S < 65536 && t * Hkv < (1LL << 26), "od_kv_append_i8: too many states or tokens in one call");
  const int threads = 256;
  const dim3 blocks(static_cast<unsigned>((t * Hkv * 32 + threads - 1) / threads), static_cast<unsigned>(S));
  // 8-byte loads / 4-byte stores per lane when every row start allows them (element strides multiples of 4)
  const auto a = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
  const bool vec = a(k, 8) && a(v, 8) && a(kq, 4) && a(vq, 4) && ks_s % 4 == 0 && ks_t % 4 == 0 && ks_h % 4 == 0 &&
                   vs_s % 4 == 0 && vs_t % 4 == 0 && vs_h % 4 == 0;
#define OD_KV(T_, E)                                                                                           \
  kv_append_kernel<T_, E><<<blocks, threads, 0, st>>>(static_cast<const T_*>(k), static_cast<const T_*>(v), S, t, \
                                                      Hkv, ks_s, ks_t, ks_h, vs_s, vs_t, vs_h, kq, vq,          \
                                                      static_cast<T_*>(ksc), static_cast<T_*>(vsc),            \
                                                      static_cast<T_*>(kb), static_cast<T_*>(vb), T_cap, t0, vec)
  if (kv_dtype == OD_BF16) {
    if (D == 64) OD_KV(__nv_bfloat16, 2); else if (D == 128) OD_KV(__nv_bfloat16, 4); else OD_KV(__nv_bfloat16, 8);
  } else if (kv_dtype == OD_F16) {
    if (D == 64) OD_KV(__half, 2); else if (D == 128) OD_KV(__half, 4); else OD_KV(__half, 8);
  } else if (kv_dtype == OD_F32) {
    if (D == 64) OD_KV(float, 2); else if (D == 128) OD_KV(float, 4); else OD_KV(float, 8);
  } else {
    return fail(OD_EINVAL, "od_kv_append_i8: bad dtype %d", kv_dtype);
  }
#undef OD_KV
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_rmsnorm_res_quant(const void* x, const void* res_in, void* res_out, const void* w, const void* inv_s,
                                    float eps, int64_t M, int H, void* y_out, int8_t* q, float* s, void* stream) {
  OD_REQUIRE(x && w, "od_rmsnorm_res_quant: null pointer");
  OD_REQUIRE(!res_in || res_out, "od_rmsnorm_res_quant: res_in needs res_out");
  OD_REQUIRE((q == nullptr) == (s == nullptr), "od_rmsnorm_res_quant: q and s go together");
  OD_REQUIRE(y_out || q, "od_rmsnorm_res_quant: nothing to write");
  OD_REQUIRE(M >= 0 && H > 0 && H % 8 == 0, "od_rmsnorm_res_quant: bad shape M=%lld H=%d", (long long)M, H);
  OD_REQUIRE(aligned16(x) && aligned16(w) && (!res_in || (aligned16(res_in) && aligned16(res_out))) &&
             (!y_out || aligned16(y_out)) && (!q || aligned16(q)) && (!inv_s || aligned16(inv_s)),
             "od_rmsnorm_res_quant: pointers must be 16-byte aligned");
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const int vecs = (H / 8 + kRowThreads - 1) / kRowThreads;
  dim3 grid(static_cast<unsigned>(M)), block(kRowThreads);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto RI = static_cast<const __nv_bfloat16*>(res_in);
  auto RO = static_cast<__nv_bfloat16*>(res_out);
  auto Wt = static_cast<const __nv_bfloat16*>(w);
  auto IS = static_cast<const __nv_bfloat16*>(inv_s);
  auto Y = static_cast<__nv_bfloat16*>(y_out);
#define OD_RN(V) rmsnorm_res_quant_kernel<V><<<grid, block, 0, st>>>(X, RI, RO, Wt, IS, eps, H, Y, q, s)
  if (vecs <= 1) OD_RN(1);
  else if (vecs <= 2) OD_RN(2);
  else if (vecs <= 3) OD_RN(3);
  else if (vecs <= 4) OD_RN(4);
  else if (vecs <= 6) OD_RN(6);
  else if (vecs <= 8) OD_RN(8);
  else if (vecs <= 16) OD_RN(16);
  else return fail(OD_EUNSUPPORTED, "od_rmsnorm_res_quant: H=%d above %d", H, 16 * 8 * kRowThreads);
#undef OD_RN
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_embed_i8(const int64_t* ids, int64_t n, const int8_t* qweight, const void* scale, int64_t V, int H,
                           void* out, void* stream) {
  OD_REQUIRE(ids && qweight && scale && out, "od_embed_i8: null pointer");
  OD_REQUIRE(n >= 0 && V > 0 && H > 0 && H % 8 == 0, "od_embed_i8: bad shape");
  OD_REQUIRE(aligned16(out) && (reinterpret_cast<uintptr_t>(qweight) & 7) == 0, "od_embed_i8: misaligned pointers");
  if (n == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_embed_i8: no device error word");
  embed_i8_kernel<<<static_cast<unsigned>(n), 128, 0, as_stream(stream)>>>(
      ids, qweight, static_cast<const __nv_bfloat16*>(scale), V, H, static_cast<__nv_bfloat16*>(out), err);
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_gate_quant(const void* o, const void* qkv, int64_t ldqkv, int64_t M, int Hq, int D,
                             const void* inv_s, int8_t* q, float* s, void* stream) {
  OD_REQUIRE(o && qkv && q && s, "od_gate_quant: null pointer");
  OD_REQUIRE(M >= 0 && Hq > 0 && D % 8 == 0 && ldqkv % 8 == 0 && ldqkv >= 2LL * Hq * D, "od_gate_quant: bad shape");
  OD_REQUIRE(aligned16(o) && aligned16(qkv) && aligned16(q) && (!inv_s || aligned16(inv_s)),
             "od_gate_quant: pointers must be 16-byte aligned");
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const int W = Hq * D;
  const int vecs = (W / 8 + kRowThreads - 1) / kRowThreads;
  dim3 grid(static_cast<unsigned>(M)), block(kRowThreads);
  auto O = static_cast<const __nv_bfloat16*>(o);
  auto G = static_cast<const __nv_bfloat16*>(qkv);
  auto IS = static_cast<const __nv_bfloat16*>(inv_s);
#define OD_GQ(V) gate_quant_kernel<V><<<grid, block, 0, st>>>(O, G, ldqkv, Hq, D, IS, q, s)
  if (vecs <= 1) OD_GQ(1);
  else if (vecs <= 2) OD_GQ(2);
  else if (vecs <= 3) OD_GQ(3);
  else if (vecs <= 4) OD_GQ(4);
  else if (vecs <= 6) OD_GQ(6);
  else if (vecs <= 8) OD_GQ(8);
  else if (vecs <= 16) OD_GQ(16);
  else return fail(OD_EUNSUPPORTED, "od_gate_quant: Hq*D=%d above %d", W, 16 * 8 * kRowThreads);
#undef OD_GQ
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_swiglu_quant(const void* g, const void* u, int64_t M, int64_t F, const void* inv_s, int8_t* q,
                               float* s, void* stream) {
  OD_REQUIRE(g && u && q && s, "od_swiglu_quant: null pointer");
  OD_REQUIRE(M >= 0 && F > 0 && F % 8 == 0, "od_swiglu_quant: bad shape (F %% 8 == 0)");
  OD_REQUIRE(aligned16(g) && aligned16(u) && aligned16(q) && (!inv_s || aligned16(inv_s)),
             "od_swiglu_quant: pointers must be 16-byte aligned");
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const int64_t vecs = (F / 8 + kRowThreads - 1) / kRowThreads;
  dim3 grid(static_cast<unsigned>(M)), block(kRowThreads);
  auto Gp = static_cast<const __nv_bfloat16*>(g);
  auto Up = static_cast<const __nv_bfloat16*>(u);
  auto IS = static_cast<const __nv_bfloat16*>(inv_s);
#define OD_SQ(V) swiglu_quant_kernel<V><<<grid, block, 0, st>>>(Gp, Up, F, IS, q, s)
  if (vecs <= 1) OD_SQ(1);
  else if (vecs <= 2) OD_SQ(2);
  else if (vecs <= 4) OD_SQ(4);
  else if (vecs <= 6) OD_SQ(6);
  else if (vecs <= 8) OD_SQ(8);
  else if (vecs <= 12) OD_SQ(12);
  else return fail(OD_EUNSUPPORTED, "od_swiglu_quant: F=%lld above %d", (long long)F, 12 * 8 * kRowThreads);
#undef OD_SQ
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_readout(const float* logits, const float* T, const float* bias, const uint8_t* mask,
                          const int32_t* none_col, int64_t N, int64_t K, float* probs, double* renorm, float* p_none,
                          void* stream) {
  OD_REQUIRE(logits && T && mask && probs, "od_readout: null pointer");
  OD_REQUIRE(N >= 0 && K > 0, "od_readout: bad shape");
  if (N == 0) return ok();
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((N * 32 + threads - 1) / threads);
  readout_kernel<<<blocks, threads, 0, as_stream(stream)>>>(logits, T, bias, mask, none_col, N, K, probs, renorm, p_none);
  OD_LAUNCH_CHECK();
  return ok();
}
