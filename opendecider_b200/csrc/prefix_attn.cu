// Branched shared-prefix attention over an int8 state KV cache (Hydragen split of prefix_attn._split_attention,
// merged exactly by log-sum-exp, written here as one online softmax over the three key segments).
//
// One CTA = one query row r, one KV head g, 64 query slots (tokens x the GQA group's heads, like the reference's
// wide kernel rows). 4 warps, each owns 16 query slots and keeps its Q fragments and O accumulator in registers.
// Key blocks of 64 are staged in shared memory:
//   segment 1  int8 state prefix of the row's state: 16-byte vector loads of K/V bytes + per-token scales,
//              dequantised in shared memory exactly as materialize() rounds (no bf16 copy of the cache in HBM);
//   segment 2  optional bf16 question prefix (the question cache's second level);
//   segment 3  the row's own keys, causal.
// Scores and P.V run on bf16 tensor-core MMAs with fp32 accumulation; the softmax is online in the exp2 domain.
// Every row sees the same key order whatever its index, so outputs do not depend on row order.
#include <type_traits>

#include "common.cuh"

namespace od {
namespace {

constexpr int kWarps = 4;
constexpr int BM = 16 * kWarps;  // query slots per CTA
constexpr int BN = 64;           // keys per block
constexpr int kThreads = 32 * kWarps;
template <int D> constexpr int smem_bytes() { return BM * D * 2 + 2 * BN * D * 2 + BN * 4 + 128; }

// 16-byte chunk c of row `row` (rows of D bf16) lives at chunk c ^ (row & 7): ldmatrix of 8 rows is conflict-free
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct Params {
  const __nv_bfloat16* q;
  const int8_t* Kp;
  const int8_t* Vp;
  const void* ksc;
  const void* vsc;
  const int32_t* row_state;
  const int32_t* p_lo;
  const int32_t* p_hi;
  const uint8_t* pmask;
  const __nv_bfloat16* Kq;
  const __nv_bfloat16* Vq;
  const int32_t* row_q;
  const int32_t* q_len;
  const __nv_bfloat16* k_own;
  const __nv_bfloat16* v_own;
  const int32_t* own_lo;
  const int32_t* own_hi;
  __nv_bfloat16* o;
  float* lse;
  int64_t R, t, S, T, NQ, Lq;
  int Hq, Hkv, rep, tiles_per_row;
  float scale_log2;
};

// Per-warp online-softmax state: rows (lane/4) and (lane/4 + 8) of the warp's 16 slots.
template <int D>
struct Softmax {
  float m[2], l[2];
  float o[D / 8][4];
};

// S = Q K^T for one 64-key block (keys in sK), masked by `bias` (0 / -inf per key) and the causal rule, then the
// online-softmax update and O += P V (values in sV).
template <int D, bool CAUSAL>
__device__ __forceinline__ void attend_block(Softmax<D>& st, const uint32_t (&qf)[D / 16][4], uint32_t sK, uint32_t sV,
                                             const float* bias, float scale_log2, int key0, const int (&qtok)[2],
                                             int lane) {
  float s[BN / 8][4];
#pragma unroll
  for (int nt = 0; nt < BN / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
  for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
    for (int kd = 0; kd < D / 16; kd += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sK + swz<D>(nt * 8 + (lane & 7), 2 * kd + (lane >> 3)), b0, b1, b2, b3);
      mma_bf16(s[nt], qf[kd], b0, b1);
      mma_bf16(s[nt], qf[kd + 1], b2, b3);
    }
  }
  // scale, mask, block row max
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = nt * 8 + 2 * (lane & 3) + (j & 1);
      float v = s[nt][j] * scale_log2 + bias[key];
      if (CAUSAL && key0 + key > qtok[j >> 1]) v = -INFINITY;
      s[nt][j] = v;
      mx[j >> 1] = fmaxf(mx[j >> 1], v);
    }
  }
  float alpha[2], msafe[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float mn = fmaxf(st.m[h], mx[h]);
    msafe[h] = mn == -INFINITY ? 0.f : mn;
    alpha[h] = exp2f(st.m[h] - msafe[h]);
    st.m[h] = mn;
  }
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int nt = 0; nt < BN / 8; ++nt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p = exp2f(s[nt][j] - msafe[j >> 1]);
      s[nt][j] = p;
      rs[j >> 1] += p;
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) st.l[h] = st.l[h] * alpha[h] + rs[h];
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    st.o[dt][0] *= alpha[0];
    st.o[dt][1] *= alpha[0];
    st.o[dt][2] *= alpha[1];
    st.o[dt][3] *= alpha[1];
  }
  // O += P V: the S accumulator layout is the A-operand layout of the next MMA (keys = k dimension)
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    uint32_t pa[4];
    pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
    pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
    pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
    pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
    for (int dt = 0; dt < D / 8; dt += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sV + swz<D>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dt + (lane >> 4)), b0, b1, b2, b3);
      mma_bf16(st.o[dt], pa, b0, b1);
      mma_bf16(st.o[dt + 1], pa, b2, b3);
    }
  }
}

// Stage 64 int8 keys+values (rows of kD bytes) dequantised to bf16 into the swizzled tiles; invalid keys -> 0.
template <typename TS, int D>
__device__ __forceinline__ void stage_int8_block(uint8_t* sK, uint8_t* sV, float* bias, const int8_t* Kb,
                                                 const int8_t* Vb, const TS* ksc, const TS* vsc, const uint8_t* pm,
                                                 int p0, int p_hi) {
  // 64 keys x D bytes = 64 * D / 16 chunks of 16 int8 per matrix
  constexpr int CPR = D / 16;  // chunks per key row
#pragma unroll
  for (int it = 0; it < BN * CPR / kThreads; ++it) {
    const int c = threadIdx.x + it * kThreads;
    const int key = c / CPR, ch = c % CPR;
    const int p = p0 + key;
    const bool in = p < p_hi;
    int4 kraw = make_int4(0, 0, 0, 0), vraw = make_int4(0, 0, 0, 0);
    float ks = 0.f, vs = 0.f;
    if (in) {
      kraw = *reinterpret_cast<const int4*>(Kb + static_cast<int64_t>(p) * D + ch * 16);
      vraw = *reinterpret_cast<const int4*>(Vb + static_cast<int64_t>(p) * D + ch * 16);
      ks = Elem<TS>::to_f(ksc[p]);
      vs = Elem<TS>::to_f(vsc[p]);
    }
    const int8_t* kb = reinterpret_cast<const int8_t*>(&kraw);
    const int8_t* vb = reinterpret_cast<const int8_t*>(&vraw);
    // materialize(): q.to(dtype) * scale.to(dtype) rounds once to the scale dtype, then .to(bf16)
    uint32_t kw[8], vw[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float k0 = static_cast<float>(kb[2 * e]) * ks, k1 = static_cast<float>(kb[2 * e + 1]) * ks;
      float v0 = static_cast<float>(vb[2 * e]) * vs, v1 = static_cast<float>(vb[2 * e + 1]) * vs;
      if (std::is_same<TS, __half>::value) {
        k0 = rhf(k0); k1 = rhf(k1); v0 = rhf(v0); v1 = rhf(v1);
      }
      kw[e] = pack_bf16(k0, k1);
      vw[e] = pack_bf16(v0, v1);
    }
    // a 16-int8 chunk becomes two 16-byte bf16 chunks (2*ch, 2*ch + 1) of the row
    *reinterpret_cast<uint4*>(sK + swz<D>(key, 2 * ch)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
    *reinterpret_cast<uint4*>(sK + swz<D>(key, 2 * ch + 1)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
    *reinterpret_cast<uint4*>(sV + swz<D>(key, 2 * ch)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    *reinterpret_cast<uint4*>(sV + swz<D>(key, 2 * ch + 1)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    if (ch == 0) bias[key] = (in && (!pm || pm[p])) ? 0.f : -INFINITY;
  }
}

// Stage 64 bf16 keys+values; key j of the block is row (j0 + j) at stride `ld` elements; keys outside [lo, n) are
// invalid (zero-filled and masked).
template <int D>
__device__ __forceinline__ void stage_bf16_block(uint8_t* sK, uint8_t* sV, float* bias, const __nv_bfloat16* Kb,
                                                 const __nv_bfloat16* Vb, int64_t ld, int j0, int lo, int n) {
  // 64 keys x D/8 chunks of 8 bf16 per matrix
  constexpr int CPR = D / 8;
#pragma unroll
  for (int it = 0; it < BN * CPR / kThreads; ++it) {
    const int c = threadIdx.x + it * kThreads;
    const int key = c / CPR, ch = c % CPR;
    const int j = j0 + key;
    const bool in = j >= lo && j < n;
    uint4 kraw = make_uint4(0, 0, 0, 0), vraw = make_uint4(0, 0, 0, 0);
    if (in) {
      kraw = *reinterpret_cast<const uint4*>(Kb + j * ld + ch * 8);
      vraw = *reinterpret_cast<const uint4*>(Vb + j * ld + ch * 8);
    }
    *reinterpret_cast<uint4*>(sK + swz<D>(key, ch)) = kraw;
    *reinterpret_cast<uint4*>(sV + swz<D>(key, ch)) = vraw;
    if (ch == 0) bias[key] = in ? 0.f : -INFINITY;
  }
}

template <typename TS, int D>
__global__ void __launch_bounds__(kThreads) prefix_attn_kernel(Params P) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int CPR = D / 8;  // 16-byte chunks per bf16 row
  uint8_t* sQ = smem;
  uint8_t* sK = smem + BM * D * 2;
  uint8_t* sV = sK + BN * D * 2;
  float* bias = reinterpret_cast<float*>(sV + BN * D * 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x % P.tiles_per_row;
  const int64_t r = blockIdx.x / P.tiles_per_row;
  const int g = blockIdx.y;
  const int rep = P.rep;
  const int tok_per_tile = BM / rep;
  const int i0 = tile * tok_per_tile;

  // ---- Q tile: slot = (i - i0) * rep + hh  ->  q[r, i, g*rep + hh, :]
  for (int c = threadIdx.x; c < BM * CPR; c += kThreads) {
    const int slot = c / CPR, ch = c % CPR;
    const int i = i0 + slot / rep, hh = slot % rep;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < P.t) v = *reinterpret_cast<const uint4*>(P.q + ((r * P.t + i) * P.Hq + g * rep + hh) * D + ch * 8);
    *reinterpret_cast<uint4*>(sQ + swz<D>(slot, ch)) = v;
  }
  __syncthreads();
  uint32_t qf[D / 16][4];
  const uint32_t sQa = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const uint32_t sKa = static_cast<uint32_t>(__cvta_generic_to_shared(sK));
  const uint32_t sVa = static_cast<uint32_t>(__cvta_generic_to_shared(sV));
#pragma unroll
  for (int kd = 0; kd < D / 16; ++kd)
    ldsm_x4(sQa + swz<D>(warp * 16 + (lane & 15), 2 * kd + (lane >> 4)), qf[kd][0], qf[kd][1], qf[kd][2], qf[kd][3]);

  Softmax<D> st;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) st.o[dt][0] = st.o[dt][1] = st.o[dt][2] = st.o[dt][3] = 0.f;
  // query token of this thread's two rows
  const int slot_a = warp * 16 + (lane >> 2);
  const int qtok[2] = {i0 + slot_a / rep, i0 + (slot_a + 8) / rep};

  // ---- segment 1: int8 state prefix
  if (P.Kp) {
    const int stt = P.row_state[r];
    const int lo = P.p_lo ? P.p_lo[stt] : 0;
    const int hi = P.p_hi ? P.p_hi[stt] : static_cast<int>(P.T);
    const int64_t base = (static_cast<int64_t>(stt) * P.Hkv + g) * P.T;
    const int8_t* Kb = P.Kp + base * D;
    const int8_t* Vb = P.Vp + base * D;
    const TS* ks = static_cast<const TS*>(P.ksc) + base;
    const TS* vs = static_cast<const TS*>(P.vsc) + base;
    const uint8_t* pm = P.pmask ? P.pmask + static_cast<int64_t>(stt) * P.T : nullptr;
    for (int p0 = lo; p0 < hi; p0 += BN) {
      stage_int8_block<TS, D>(sK, sV, bias, Kb, Vb, ks, vs, pm, p0, hi);
      __syncthreads();
      attend_block<D, false>(st, qf, sKa, sVa, bias, P.scale_log2, 0, qtok, lane);
      __syncthreads();
    }
  }
  // ---- segment 2: bf16 question prefix
  if (P.Kq) {
    const int qr = P.row_q[r];
    const int n = P.q_len[qr];
    const int64_t ld = static_cast<int64_t>(P.Hkv) * D;
    const __nv_bfloat16* Kb = P.Kq + (static_cast<int64_t>(qr) * P.Lq * P.Hkv + g) * D;
    const __nv_bfloat16* Vb = P.Vq + (static_cast<int64_t>(qr) * P.Lq * P.Hkv + g) * D;
    for (int j0 = 0; j0 < n; j0 += BN) {
      stage_bf16_block<D>(sK, sV, bias, Kb, Vb, ld, j0, 0, n);
      __syncthreads();
      attend_block<D, false>(st, qf, sKa, sVa, bias, P.scale_log2, 0, qtok, lane);
      __syncthreads();
    }
  }
  // ---- segment 3: own keys, causal
  {
    const int lo = P.own_lo ? P.own_lo[r] : 0;
    const int n = P.own_hi ? P.own_hi[r] : static_cast<int>(P.t);
    const int last = min(static_cast<int>(P.t), i0 + tok_per_tile);  // keys past the tile's last token are never visible
    const int64_t ld = static_cast<int64_t>(P.Hkv) * D;
    const __nv_bfloat16* Kb = P.k_own + (r * P.t * P.Hkv + g) * D;
    const __nv_bfloat16* Vb = P.v_own + (r * P.t * P.Hkv + g) * D;
    for (int j0 = (lo / BN) * BN; j0 < last; j0 += BN) {
      stage_bf16_block<D>(sK, sV, bias, Kb, Vb, ld, j0, lo, min(n, last));
      __syncthreads();
      attend_block<D, true>(st, qf, sKa, sVa, bias, P.scale_log2, j0, qtok, lane);
      __syncthreads();
    }
  }

  // ---- finalise: O / l, natural-log LSE
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    st.l[h] += __shfl_xor_sync(0xffffffffu, st.l[h], 1);
    st.l[h] += __shfl_xor_sync(0xffffffffu, st.l[h], 2);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int slot = slot_a + 8 * h;
    const int i = i0 + slot / rep, hh = slot % rep;
    if (i >= P.t) continue;
    const float inv = st.l[h] == 0.f ? 0.f : 1.0f / st.l[h];
    __nv_bfloat16* dst = P.o + ((r * P.t + i) * P.Hq + g * rep + hh) * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      const int d = dt * 8 + 2 * (lane & 3);
      *reinterpret_cast<__nv_bfloat162*>(dst + d) =
          __floats2bfloat162_rn(st.o[dt][2 * h] * inv, st.o[dt][2 * h + 1] * inv);
    }
    if (P.lse && (lane & 3) == 0)
      P.lse[(r * P.Hq + g * rep + hh) * P.t + i] =
          st.l[h] == 0.f ? -INFINITY : (st.m[h] + log2f(st.l[h])) * 0.6931471805599453f;
  }
}

template <typename TS, int D>
int launch_attn(const Params& P, dim3 grid, cudaStream_t st) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(prefix_attn_kernel<TS, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     smem_bytes<D>()));
    attr[dev] = true;
  }
  prefix_attn_kernel<TS, D><<<grid, kThreads, smem_bytes<D>(), st>>>(P);
  OD_LAUNCH_CHECK();
  return ok();
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_prefix_attn(const void* q, const int8_t* Kp, const int8_t* Vp, const void* ksc, const void* vsc,
                              const int32_t* row_state, const int32_t* p_lo, const int32_t* p_hi, const uint8_t* pmask,
                              const void* Kq, const void* Vq, const int32_t* row_q, const int32_t* q_len,
                              const void* k_own, const void* v_own, const int32_t* own_lo, const int32_t* own_hi,
                              void* o, float* lse,
                              od_attn_dims dims, void* stream) {
  OD_REQUIRE(q && k_own && v_own && o, "od_prefix_attn: null pointer");
  OD_REQUIRE(dims.D == 64 || dims.D == 128, "od_prefix_attn: head_dim %d not in {64, 128}", dims.D);
  OD_REQUIRE(dims.Hq > 0 && dims.Hkv > 0 && dims.Hq % dims.Hkv == 0, "od_prefix_attn: bad head counts");
  const int rep = dims.Hq / dims.Hkv;
  OD_REQUIRE(BM % rep == 0, "od_prefix_attn: GQA group %d does not divide %d", rep, BM);
  OD_REQUIRE(dims.R >= 0 && dims.t >= 0 && dims.t < (1 << 30), "od_prefix_attn: bad R/t");
  OD_REQUIRE(!Kp || (Vp && ksc && vsc && row_state && dims.S > 0 && dims.T > 0 && dims.T < (1 << 30)),
             "od_prefix_attn: the int8 prefix needs Vp, scales, row_state, S, T");
  OD_REQUIRE(!Kp || dims.scale_dtype == OD_BF16 || dims.scale_dtype == OD_F16, "od_prefix_attn: scale dtype");
  OD_REQUIRE(!Kq || (Vq && row_q && q_len && dims.NQ > 0 && dims.Lq > 0), "od_prefix_attn: bad question prefix");
  OD_REQUIRE(aligned16(q) && aligned16(k_own) && aligned16(v_own) && (!Kp || (aligned16(Kp) && aligned16(Vp))) &&
                 (!Kq || (aligned16(Kq) && aligned16(Vq))),
             "od_prefix_attn: tensors must be 16-byte aligned");
  if (dims.R == 0 || dims.t == 0) return ok();
  Params P;
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.Kp = Kp;
  P.Vp = Vp;
  P.ksc = ksc;
  P.vsc = vsc;
  P.row_state = row_state;
  P.p_lo = p_lo;
  P.p_hi = p_hi;
  P.pmask = pmask;
  P.Kq = static_cast<const __nv_bfloat16*>(Kq);
  P.Vq = static_cast<const __nv_bfloat16*>(Vq);
  P.row_q = row_q;
  P.q_len = q_len;
  P.k_own = static_cast<const __nv_bfloat16*>(k_own);
  P.v_own = static_cast<const __nv_bfloat16*>(v_own);
  P.own_lo = own_lo;
  P.own_hi = own_hi;
  P.o = static_cast<__nv_bfloat16*>(o);
  P.lse = lse;
  P.R = dims.R; P.t = dims.t; P.S = dims.S; P.T = dims.T; P.NQ = dims.NQ; P.Lq = dims.Lq;
  P.Hq = dims.Hq; P.Hkv = dims.Hkv; P.rep = rep;
  P.tiles_per_row = static_cast<int>((dims.t * rep + BM - 1) / BM);
  P.scale_log2 = dims.sm_scale * 1.4426950408889634f;
  const int64_t gx = dims.R * P.tiles_per_row;
  OD_REQUIRE(gx < (1LL << 31) && dims.Hkv < 65536, "od_prefix_attn: grid too large");
  dim3 grid(static_cast<unsigned>(gx), dims.Hkv);
  cudaStream_t st = as_stream(stream);
  const bool half_scale = Kp && dims.scale_dtype == OD_F16;
  if (dims.D == 128) {
    if (half_scale) return launch_attn<__half, 128>(P, grid, st);
    return launch_attn<__nv_bfloat16, 128>(P, grid, st);
  }
  if (half_scale) return launch_attn<__half, 64>(P, grid, st);
  return launch_attn<__nv_bfloat16, 64>(P, grid, st);
}
