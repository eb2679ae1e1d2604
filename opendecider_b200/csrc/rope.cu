// Attention pre-processing on the fused q/k/v projection output: gated-q split, per-head q/k RMSNorm (1 + w) and
// rotate-half RoPE, with the rounding points of the bf16 reference (Qwen3_5Attention.forward, prefix_attn._forward),
// optionally with the int8 KV-cache write of the pass's k / v heads in the same kernel (the state pass, appended
// records). Bandwidth-bound: every input read once, every output written once, in 16-byte vectors.
#include "common.cuh"

namespace od {
namespace {

constexpr int kWarps = 2;              // small CTAs, 16 per SM: more tokens' loads in flight per SM

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

// The kernel: 16-byte vectors. A head of D elements is handled by D / 8 lanes ("a head unit", 8 elements per lane: one
// 16-byte load and store); rotate_half's partner element (d +- D/2) sits D/16 lanes away in the same unit. A CTA of
// kWarps warps has kWarps * 256 / D head units and handles kTokensPerCta consecutive tokens; unit u takes the token's
// head slots u, u + units, ... with the loads of kUnroll slots issued before their math.
constexpr int kTokensPerCta = 4;
constexpr int kUnroll = 3;

// the KV-cache row of a k / v head held by a head unit (8 values per lane): per (state, head, token) int8 over D as
// od_kv_append_i8 does it, the scale in bf16, and optionally the materialised bf16 copy
template <int LPH>
__device__ __forceinline__ void write_kv_unit(const uint4& w, int8_t* q8, __nv_bfloat16* sc, __nv_bfloat16* mat,
                                              int64_t dst, int li, uint32_t umask) {
  constexpr int D = LPH * 8;
  float x[8];
  unpack8(w, x);
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(umask, amax, o));
  const float s = quant_scale(amax), r = quant_recip(s);
  const uint2 qw = quant8(x, s, r);
  *reinterpret_cast<uint2*>(q8 + dst * D + li * 8) = qw;
  const __nv_bfloat16 sb = __float2bfloat16_rn(s);
  if (li == 0) sc[dst] = sb;
  if (mat != nullptr) {                              // bf16(q * s): exact products (|q| <= 127, s has 8 bits)
    const uint32_t s2 = static_cast<uint32_t>(__bfloat16_as_ushort(sb)) * 0x10001u;
    uint32_t m[4];
    dequant4_bf16(qw.x, s2, m[0], m[1]);
    dequant4_bf16(qw.y, s2, m[2], m[3]);
    *reinterpret_cast<uint4*>(mat + dst * D + li * 8) = make_uint4(m[0], m[1], m[2], m[3]);
  }
}

template <int D, bool KV>
__global__ void __launch_bounds__(32 * kWarps, 16) qk_norm_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, int64_t ld, const int32_t* __restrict__ pos,
    const __nv_bfloat16* __restrict__ cos_t, const __nv_bfloat16* __restrict__ sin_t, int64_t P,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps, int64_t M, int Hq, int Hkv,
    __nv_bfloat16* __restrict__ qo, __nv_bfloat16* __restrict__ ko, __nv_bfloat16* __restrict__ vo, int32_t* err,
    KvOut kv) {
  constexpr int LPH = D / 8;                          // lanes per head unit
  constexpr int kUnits = kWarps * 32 / LPH;
  const int unit = threadIdx.x / LPH, li = threadIdx.x % LPH;
  // the head unit's lanes: its shuffles name only them (units of one warp may take different branches)
  const uint32_t umask = (LPH == 32 ? 0xffffffffu : ((1u << LPH) - 1u)) << ((threadIdx.x & 31) & ~(LPH - 1));
  const int slots = Hq + 2 * Hkv;
  // this lane's 8 elements of the (1 + w) norm factors, fp32 (Qwen3_5RMSNorm's weight offset)
  float2 q1[4], k1[4];
  {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(qw + li * 8));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(kw + li * 8));
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      q1[e] = __fadd2_rn(make_float2(1.0f, 1.0f), unpack2(aw[e]));
      k1[e] = __fadd2_rn(make_float2(1.0f, 1.0f), unpack2(bw[e]));
    }
  }
  const uint32_t neg = li < LPH / 2 ? 0x80008000u : 0u;  // rotate_half negates the first half's partners
  const int64_t tok_end = min(M, static_cast<int64_t>(blockIdx.x + 1) * kTokensPerCta);
  for (int64_t tok = static_cast<int64_t>(blockIdx.x) * kTokensPerCta; tok < tok_end; ++tok) {
    const __nv_bfloat16* row = qkv + tok * ld;
    int p = pos[tok];
    if (p < 0 || p >= P) {
      if (threadIdx.x == 0) atomicCAS(err, 0, 0x7E0000 | 1);
      p = 0;
    }
    const uint4 cv = __ldg(reinterpret_cast<const uint4*>(cos_t + static_cast<int64_t>(p) * D + li * 8));
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sin_t + static_cast<int64_t>(p) * D + li * 8));
    const uint32_t c[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
    int kv_r = 0, kv_j = 0;                            // cache position of this token (fused KV write)
    if constexpr (KV) {
      kv_r = static_cast<int>(tok / kv.t);
      kv_j = static_cast<int>(tok - static_cast<int64_t>(kv_r) * kv.t);
    }
    for (int s0 = unit; s0 < slots; s0 += kUnits * kUnroll) {
      // the slots' sources: q head h at h * 2D (its gate follows), k head at Hq * 2D + h * D, v head after the k heads
      uint4 x[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int slot = s0 + u * kUnits;
        if (slot < slots) {
          const int64_t off = slot < Hq ? static_cast<int64_t>(slot) * 2 * D
                                        : static_cast<int64_t>(Hq) * 2 * D + static_cast<int64_t>(slot - Hq) * D;
          x[u] = __ldg(reinterpret_cast<const uint4*>(row + off + li * 8));
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int slot = s0 + u * kUnits;
        if (slot >= slots) break;                      // uniform across the head unit
        if (slot >= Hq + Hkv) {                        // value head: plain copy (+ its cache row)
          const int h = slot - Hq - Hkv;
          *reinterpret_cast<uint4*>(vo + (tok * Hkv + h) * D + li * 8) = x[u];
          if constexpr (KV)
            write_kv_unit<LPH>(x[u], kv.vq, kv.vsc, kv.vb,
                               (static_cast<int64_t>(kv_r) * Hkv + h) * kv.T_cap + kv.t0 + kv_j, li, umask);
          continue;
        }
        const bool is_q = slot < Hq;
        const uint32_t xw[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
        // Qwen3_5RMSNorm over the head: mean of squares in fp32 (/ D exact), y = bf16((x * rs) * (1 + w))
        float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack2(xw[e]);
          ss2 = __fadd2_rn(ss2, __fmul2_rn(f, f));
        }
        float ss = ss2.x + ss2.y;
#pragma unroll
        for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(umask, ss, o);
        const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / D), eps)));
        const float2 rs2 = make_float2(rs, rs);
        uint32_t y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 v = __fmul2_rn(__fmul2_rn(unpack2(xw[e]), rs2), is_q ? q1[e] : k1[e]);
          y[e] = pack_rn(v.x, v.y);
        }
        // RoPE: q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16
        uint32_t r[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t rh = __shfl_xor_sync(umask, y[e], LPH / 2) ^ neg;
          r[e] = badd2(bmul2(y[e], c[e]), bmul2(rh, sn[e]));
        }
        const uint4 out = make_uint4(r[0], r[1], r[2], r[3]);
        __nv_bfloat16* dst = is_q ? qo + (tok * Hq + slot) * D : ko + (tok * Hkv + (slot - Hq)) * D;
        *reinterpret_cast<uint4*>(dst + li * 8) = out;
        if constexpr (KV) {
          if (!is_q)
            write_kv_unit<LPH>(out, kv.kq, kv.ksc, kv.kb,
                               (static_cast<int64_t>(kv_r) * Hkv + (slot - Hq)) * kv.T_cap + kv.t0 + kv_j, li,
                               umask);
        }
      }
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
  OD_REQUIRE(aligned16(qkv) && aligned16(cos) && aligned16(sin) && aligned16(qnorm_w) && aligned16(knorm_w) &&
                 aligned16(q_out) && aligned16(k_out) && aligned16(v_out),
             "od_qk_norm_rope: pointers must be 16-byte aligned");
  if (M == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_qk_norm_rope: no device error word");
  const int64_t ld = static_cast<int64_t>(Hq) * 2 * D + 2LL * Hkv * D;
  OD_REQUIRE(M < (1LL << 31), "od_qk_norm_rope: too many tokens");
  const int threads = 32 * kWarps;
  const unsigned blocks = static_cast<unsigned>((M + kTokensPerCta - 1) / kTokensPerCta);
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
    if (D == 64) OD_RP(64, true);
    else if (D == 128) OD_RP(128, true);
    else OD_RP(256, true);
  } else {
    if (D == 64) OD_RP(64, false);
    else if (D == 128) OD_RP(128, false);
    else OD_RP(256, false);
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
  OD_REQUIRE(aligned16(kq) && aligned16(vq) && (kb == nullptr || (aligned16(kb) && aligned16(vb))),
             "od_qk_norm_rope_kv_i8: cache pointers must be 16-byte aligned");
  KvOut kv{kq, vq, static_cast<__nv_bfloat16*>(ksc), static_cast<__nv_bfloat16*>(vsc),
           static_cast<__nv_bfloat16*>(kb), static_cast<__nv_bfloat16*>(vb), t, T_cap, t0};
  return launch_qk_norm_rope(qkv, pos, cos, sin, P, qnorm_w, knorm_w, eps, M, Hq, Hkv, D, q_out, k_out, v_out, &kv,
                             stream);
}
