// Attention pre-processing on the fused q/k/v projection output: gated-q split, per-head q/k RMSNorm (1 + w) and
// rotate-half RoPE, with the rounding points of the bf16 reference (Qwen3_5Attention.forward, prefix_attn._forward).
// One warp per (token, head slot); each lane holds D/32 contiguous elements, so rotate_half's partner element
// (d +- D/2) sits in lane ^ 16 and is exchanged with one shuffle.
#include "common.cuh"

namespace od {
namespace {

template <int EPL>
__device__ __forceinline__ void load_lane(const __nv_bfloat16* p, float (&x)[EPL]) {
  if constexpr (EPL == 4) {
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = __bfloat162float(p[i]);
  }
}
template <int EPL>
__device__ __forceinline__ void store_lane(__nv_bfloat16* p, const float (&x)[EPL]) {
  if constexpr (EPL == 4) {
    uint2 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
    h[0] = __floats2bfloat162_rn(x[0], x[1]);
    h[1] = __floats2bfloat162_rn(x[2], x[3]);
    *reinterpret_cast<uint2*>(p) = raw;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = __float2bfloat16_rn(x[i]);
  }
}

template <int EPL>
__global__ void qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld, const int32_t* __restrict__ pos,
                                    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t,
                                    int64_t P, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                    float eps, int64_t M, int Hq, int Hkv, __nv_bfloat16* __restrict__ qo,
                                    __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo, int32_t* err) {
  constexpr int D = EPL * 32;
  const int64_t item = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int slots = Hq + 2 * Hkv;
  if (item >= M * slots) return;
  const int64_t tok = item / slots;
  const int slot = static_cast<int>(item % slots);
  const __nv_bfloat16* row = qkv + tok * ld;
  float x[EPL];
  if (slot >= Hq + Hkv) {  // value head: plain copy
    const int h = slot - Hq - Hkv;
    load_lane<EPL>(row + static_cast<int64_t>(Hq) * 2 * D + static_cast<int64_t>(Hkv) * D + h * D + lane * EPL, x);
    store_lane<EPL>(vo + (tok * Hkv + h) * D + lane * EPL, x);
    return;
  }
  const bool is_q = slot < Hq;
  const int h = is_q ? slot : slot - Hq;
  const __nv_bfloat16* src = is_q ? row + static_cast<int64_t>(h) * 2 * D : row + static_cast<int64_t>(Hq) * 2 * D + h * D;
  const __nv_bfloat16* w = is_q ? qw : kw;
  load_lane<EPL>(src + lane * EPL, x);
  // Qwen3_5RMSNorm over the head dimension
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps)));
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const float wi = __bfloat162float(w[lane * EPL + i]);
    x[i] = rbf(__fmul_rn(__fmul_rn(x[i], rs), __fadd_rn(1.0f, wi)));
  }
  // RoPE: q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16
  int p = pos[tok];
  if (p < 0 || p >= P) {
    if (lane == 0) atomicCAS(err, 0, 0x7E0000 | 1);
    p = 0;
  }
  const __nv_bfloat16* c = cos_t + static_cast<int64_t>(p) * D + lane * EPL;
  const __nv_bfloat16* s = sin_t + static_cast<int64_t>(p) * D + lane * EPL;
  float y[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
    const float rh = lane < 16 ? -partner : partner;
    y[i] = rbf(rbf(x[i] * __bfloat162float(c[i])) + rbf(rh * __bfloat162float(s[i])));
  }
  __nv_bfloat16* dst = is_q ? qo + (tok * Hq + h) * D : ko + (tok * Hkv + h) * D;
  store_lane<EPL>(dst + lane * EPL, y);
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_qk_norm_rope(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                               const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv, int D,
                               void* q_out, void* k_out, void* v_out, void* stream) {
  OD_REQUIRE(qkv && pos && cos && sin && qnorm_w && knorm_w && q_out && k_out && v_out, "od_qk_norm_rope: null pointer");
  OD_REQUIRE(M >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && P > 0, "od_qk_norm_rope: bad shape");
  OD_REQUIRE(D == 64 || D == 128 || D == 256, "od_qk_norm_rope: head_dim %d not in {64, 128, 256}", D);
  if (M == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_qk_norm_rope: no device error word");
  const int64_t ld = static_cast<int64_t>(Hq) * 2 * D + 2LL * Hkv * D;
  const int64_t warps = M * (Hq + 2 * Hkv);
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((warps * 32 + threads - 1) / threads);
  cudaStream_t st = as_stream(stream);
  auto Q = static_cast<const __nv_bfloat16*>(qkv);
  auto C = static_cast<const __nv_bfloat16*>(cos);
  auto S = static_cast<const __nv_bfloat16*>(sin);
  auto QW = static_cast<const __nv_bfloat16*>(qnorm_w);
  auto KW = static_cast<const __nv_bfloat16*>(knorm_w);
  auto QO = static_cast<__nv_bfloat16*>(q_out);
  auto KO = static_cast<__nv_bfloat16*>(k_out);
  auto VO = static_cast<__nv_bfloat16*>(v_out);
#define OD_RP(E) qk_norm_rope_kernel<E><<<blocks, threads, 0, st>>>(Q, ld, pos, C, S, P, QW, KW, eps, M, Hq, Hkv, QO, KO, VO, err)
  if (D == 64) OD_RP(2);
  else if (D == 128) OD_RP(4);
  else OD_RP(8);
#undef OD_RP
  OD_LAUNCH_CHECK();
  return ok();
}
