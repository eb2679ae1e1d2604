// Attention pre-processing on the fused q/k/v projection output: gated-q split, per-head q/k RMSNorm (1 + w) and
// rotate-half RoPE, with the rounding points of the bf16 reference (Qwen3_5Attention.forward, prefix_attn._forward).
// One CTA per token, one warp per head slot at a time; each lane holds D/32 contiguous elements, so rotate_half's
// partner element (d +- D/2) sits in lane ^ 16 and is exchanged with one shuffle.
#include "common.cuh"

namespace od {
namespace {

template <int EPL>
__device__ __forceinline__ void load_lane(const __nv_bfloat16* p, float (&x)[EPL]) {
  if constexpr (EPL == 4) {
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  } else if constexpr (EPL == 2) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    x[0] = a.x; x[1] = a.y;
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

// One CTA of kWarps warps per token: the token's cos / sin rows and the two (1 + w) norm factors are loaded once
// per lane and serve all of the token's q and k heads; each warp takes head slots warp, warp + kWarps, ... and issues
// the loads of all of them before the math. A lane holds NW = EPL / 2 bf16 pairs of each head.
constexpr int kWarps = 8;
constexpr int kMaxSlotsPerWarp = 8;   // Hq + 2 Hkv <= 64

template <int EPL>
__device__ __forceinline__ void load_pairs(const __nv_bfloat16* p, uint32_t (&w)[EPL / 2]) {
  if constexpr (EPL == 4) {
    const uint2 r = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = r.x;
    w[1] = r.y;
  } else if constexpr (EPL == 8) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = r.x; w[1] = r.y; w[2] = r.z; w[3] = r.w;
  } else {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  }
}
template <int EPL>
__device__ __forceinline__ void store_pairs(__nv_bfloat16* p, const uint32_t (&w)[EPL / 2]) {
  if constexpr (EPL == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else if constexpr (EPL == 8) {
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}

// The int8 KV cache rows of a pass (state pass, appended records): token tok = row r x t + j of the pass is cache
// position t0 + j of state r. Each k / v head row is quantised per (state, head, token) over D exactly as
// od_kv_append_i8 does it (the same helpers), its scale stored in bf16, and optionally its materialised bf16 copy.
struct KvOut {
  int8_t* kq;
  int8_t* vq;
  __nv_bfloat16* ksc;
  __nv_bfloat16* vsc;
  __nv_bfloat16* kb;        // optional (with vb): bf16(q * s), materialize()'s rounding
  __nv_bfloat16* vb;
  int64_t t, T_cap, t0;
};

template <int EPL>
__device__ __forceinline__ void write_kv_row(const uint32_t (&w)[EPL / 2], int8_t* q8, __nv_bfloat16* sc,
                                             __nv_bfloat16* mat, int64_t dst, int lane) {
  constexpr int D = EPL * 32;
  float x[EPL];
#pragma unroll
  for (int e = 0; e < EPL / 2; ++e) {
    const float2 f = unpack2(w[e]);
    x[2 * e] = f.x;
    x[2 * e + 1] = f.y;
  }
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) amax = fmaxf(amax, fabsf(x[e]));
  amax = warp_max(amax);
  const float s = quant_scale(amax), r = quant_recip(s);
  int8_t qv[EPL];
  int8_t* out = q8 + dst * D + lane * EPL;
  if constexpr (EPL == 4) {
    const uint32_t word = quant4(x[0], x[1], x[2], x[3], s, r);
    *reinterpret_cast<uint32_t*>(out) = word;
#pragma unroll
    for (int e = 0; e < 4; ++e) qv[e] = static_cast<int8_t>(word >> (8 * e));
  } else if constexpr (EPL == 8) {
    const uint32_t w0 = quant4(x[0], x[1], x[2], x[3], s, r), w1 = quant4(x[4], x[5], x[6], x[7], s, r);
    *reinterpret_cast<uint2*>(out) = make_uint2(w0, w1);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qv[e] = static_cast<int8_t>(w0 >> (8 * e));
      qv[4 + e] = static_cast<int8_t>(w1 >> (8 * e));
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      qv[e] = quant_val(x[e], s, r);
      out[e] = qv[e];
    }
  }
  const __nv_bfloat16 sb = __float2bfloat16_rn(s);
  if (lane == 0) sc[dst] = sb;
  if (mat != nullptr) {
    const float sf = __bfloat162float(sb);
    float m[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) m[e] = static_cast<float>(qv[e]) * sf;   // exact: |q| <= 127, s has 8 bits
    store_lane<EPL>(mat + dst * D + lane * EPL, m);
  }
}

template <int EPL, bool KV>
__global__ void __launch_bounds__(32 * kWarps) qk_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ld, const int32_t* __restrict__ pos,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int64_t P,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps, int64_t M, int Hq, int Hkv,
    __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo, int32_t* err,
    KvOut kv) {
  constexpr int D = EPL * 32;
  constexpr int NW = EPL / 2;
  const int64_t tok = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slots = Hq + 2 * Hkv;
  const __nv_bfloat16* row = qkv + tok * ld;
  // the slot's source: q head h at h * 2D (its gate follows), k head at Hq * 2D + h * D, v head after the k heads
  uint32_t x[kMaxSlotsPerWarp][NW];
#pragma unroll
  for (int i = 0; i < kMaxSlotsPerWarp; ++i) {
    const int slot = warp + i * kWarps;
    if (slot < slots) {
      const __nv_bfloat16* src = slot < Hq ? row + static_cast<int64_t>(slot) * 2 * D
                                           : row + static_cast<int64_t>(Hq) * 2 * D + static_cast<int64_t>(slot - Hq) * D;
      load_pairs<EPL>(src + lane * EPL, x[i]);
    }
  }
  // cache position of this token (fused KV write): row r of the pass, token j, one 32-bit division per token
  int kv_r = 0, kv_j = 0;
  if constexpr (KV) {
    kv_r = static_cast<int>(tok) / static_cast<int>(kv.t);
    kv_j = static_cast<int>(tok) - kv_r * static_cast<int>(kv.t);
  }
  int p = pos[tok];
  if (p < 0 || p >= P) {
    if (threadIdx.x == 0) atomicCAS(err, 0, 0x7E0000 | 1);
    p = 0;
  }
  uint32_t c[NW], sn[NW], wq[NW], wk[NW];
  load_pairs<EPL>(cos_t + static_cast<int64_t>(p) * D + lane * EPL, c);
  load_pairs<EPL>(sin_t + static_cast<int64_t>(p) * D + lane * EPL, sn);
  load_pairs<EPL>(qw + lane * EPL, wq);
  load_pairs<EPL>(kw + lane * EPL, wk);
  float2 q1[NW], k1[NW];                              // 1 + w in fp32 (Qwen3_5RMSNorm's weight offset)
#pragma unroll
  for (int e = 0; e < NW; ++e) {
    q1[e] = __fadd2_rn(make_float2(1.0f, 1.0f), unpack2(wq[e]));
    k1[e] = __fadd2_rn(make_float2(1.0f, 1.0f), unpack2(wk[e]));
  }
  const uint32_t neg = lane < 16 ? 0x80008000u : 0u;  // rotate_half negates the first half's partners
#pragma unroll
  for (int i = 0; i < kMaxSlotsPerWarp; ++i) {
    const int slot = warp + i * kWarps;
    if (slot >= slots) break;
    if (slot >= Hq + Hkv) {                           // value head: plain copy
      const int h = slot - Hq - Hkv;
      store_pairs<EPL>(vo + (tok * Hkv + h) * D + lane * EPL, x[i]);
      if constexpr (KV)
        write_kv_row<EPL>(x[i], kv.vq, kv.vsc, kv.vb,
                          (static_cast<int64_t>(kv_r) * Hkv + h) * kv.T_cap + kv.t0 + kv_j, lane);
      continue;
    }
    const bool is_q = slot < Hq;
    // Qwen3_5RMSNorm over the head dimension: mean of squares in fp32 (/ D is exact: D is a power of two),
    // y = bf16((x * rs) * (1 + w))
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < NW; ++e) {
      const float2 f = unpack2(x[i][e]);
      ss += f.x * f.x;
      ss += f.y * f.y;
    }
    ss = warp_sum(ss);
    const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / D), eps)));
    const float2 rs2 = make_float2(rs, rs);
    uint32_t y[NW];
#pragma unroll
    for (int e = 0; e < NW; ++e) {
      const float2 v = __fmul2_rn(__fmul2_rn(unpack2(x[i][e]), rs2), is_q ? q1[e] : k1[e]);
      y[e] = pack_rn(v.x, v.y);
    }
    // RoPE: q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16; the partner element d +- D/2
    // sits in lane ^ 16
#pragma unroll
    for (int e = 0; e < NW; ++e) {
      const uint32_t rh = __shfl_xor_sync(0xffffffffu, y[e], 16) ^ neg;
      x[i][e] = badd2(bmul2(y[e], c[e]), bmul2(rh, sn[e]));
    }
    __nv_bfloat16* dst = is_q ? qo + (tok * Hq + slot) * D : ko + (tok * Hkv + (slot - Hq)) * D;
    store_pairs<EPL>(dst + lane * EPL, x[i]);
    if constexpr (KV) {
      if (!is_q)
        write_kv_row<EPL>(x[i], kv.kq, kv.ksc, kv.kb,
                          (static_cast<int64_t>(kv_r) * Hkv + (slot - Hq)) * kv.T_cap + kv.t0 + kv_j, lane);
    }
  }
}

}  // namespace
}  // namespace od

using namespace od;

namespace od {
namespace {
int launch_qk_norm_rope(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                        const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv, int D,
                        void* q_out, void* k_out, void* v_out, const KvOut* kv, void* stream) {
  OD_REQUIRE(qkv && pos && cos && sin && qnorm_w && knorm_w && q_out && k_out && v_out, "od_qk_norm_rope: null pointer");
  OD_REQUIRE(M >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && P > 0, "od_qk_norm_rope: bad shape");
  OD_REQUIRE(D == 64 || D == 128 || D == 256, "od_qk_norm_rope: head_dim %d not in {64, 128, 256}", D);
  OD_REQUIRE(aligned8(qkv) && aligned8(cos) && aligned8(sin) && aligned8(qnorm_w) && aligned8(knorm_w) &&
                 aligned8(q_out) && aligned8(k_out) && aligned8(v_out),
             "od_qk_norm_rope: pointers must be 8-byte aligned");
  if (M == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_qk_norm_rope: no device error word");
  const int64_t ld = static_cast<int64_t>(Hq) * 2 * D + 2LL * Hkv * D;
  OD_REQUIRE(Hq + 2 * Hkv <= kWarps * kMaxSlotsPerWarp, "od_qk_norm_rope: more than %d head slots",
             kWarps * kMaxSlotsPerWarp);
  OD_REQUIRE(M < (1LL << 31), "od_qk_norm_rope: too many tokens");
  const int threads = 32 * kWarps;
  const unsigned blocks = static_cast<unsigned>(M);
  cudaStream_t st = as_stream(stream);
  auto Q = static_cast<const __nv_bfloat16*>(qkv);
  auto C = static_cast<const __nv_bfloat16*>(cos);
  auto S = static_cast<const __nv_bfloat16*>(sin);
  auto QW = static_cast<const __nv_bfloat16*>(qnorm_w);
  auto KW = static_cast<const __nv_bfloat16*>(knorm_w);
  auto QO = static_cast<__nv_bfloat16*>(q_out);
  auto KO = static_cast<__nv_bfloat16*>(k_out);
  auto VO = static_cast<__nv_bfloat16*>(v_out);
  const KvOut none{};
#define OD_RP(E, KV_) qk_norm_rope_kernel<E, KV_><<<blocks, threads, 0, st>>>(Q, ld, pos, C, S, P, QW, KW, eps, M, Hq, \
                                                                              Hkv, QO, KO, VO, err, kv ? *kv : none)
  if (kv) {
    if (D == 64) OD_RP(2, true);
    else if (D == 128) OD_RP(4, true);
    else OD_RP(8, true);
  } else {
    if (D == 64) OD_RP(2, false);
    else if (D == 128) OD_RP(4, false);
    else OD_RP(8, false);
  }
#undef OD_RP
  OD_LAUNCH_CHECK();
  return ok();
}
}  // namespace
}  // namespace od

extern "C" int od_qk_norm_rope(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                               const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv, int D,
                               void* q_out, void* k_out, void* v_out, void* stream) {
  return launch_qk_norm_rope(qkv, pos, cos, sin, P, qnorm_w, knorm_w, eps, M, Hq, Hkv, D, q_out, k_out, v_out, nullptr,
                             stream);
}

extern "C" int od_qk_norm_rope_kv_i8(const void* qkv, const int32_t* pos, const void* cos, const void* sin, int64_t P,
                                     const void* qnorm_w, const void* knorm_w, float eps, int64_t M, int Hq, int Hkv,
                                     int D, void* q_out, void* k_out, void* v_out, int64_t t, int8_t* kq, int8_t* vq,
                                     void* ksc, void* vsc, void* kb, void* vb, int64_t T_cap, int64_t t0,
                                     void* stream) {
  OD_REQUIRE(kq && vq && ksc && vsc, "od_qk_norm_rope_kv_i8: null cache pointer");
  OD_REQUIRE((kb == nullptr) == (vb == nullptr), "od_qk_norm_rope_kv_i8: kb and vb go together");
  OD_REQUIRE(t > 0 && M % t == 0 && t0 >= 0 && t0 + t <= T_cap, "od_qk_norm_rope_kv_i8: bad token layout");
  OD_REQUIRE(aligned8(kq) && aligned8(vq) && (kb == nullptr || (aligned8(kb) && aligned8(vb))),
             "od_qk_norm_rope_kv_i8: cache pointers must be 8-byte aligned");
  KvOut kv{kq, vq, static_cast<__nv_bfloat16*>(ksc), static_cast<__nv_bfloat16*>(vsc),
           static_cast<__nv_bfloat16*>(kb), static_cast<__nv_bfloat16*>(vb), t, T_cap, t0};
  return launch_qk_norm_rope(qkv, pos, cos, sin, P, qnorm_w, knorm_w, eps, M, Hq, Hkv, D, q_out, k_out, v_out, &kv,
                             stream);
}
