// Branched shared-prefix attention on the sm_100a tensor cores (the Hydragen split of prefix_attn._split_attention,
// merged exactly by log-sum-exp, here as one online softmax over the three key segments of a query row).
//
// One CTA = 128 query slots (one per softmax thread and per TMEM lane) of one KV head: the slots are (row, token,
// head of the GQA group) of a row group - one long row (the state pass: 32 tokens x 4 heads per CTA) or several
// short rows of the same question (option rows), so the tensor-core tile is filled and each prefix block staged once
// serves all of them. Keys run in blocks of 64 through a warp-specialised pipeline:
//   producer warps (4)   stage K and V of block j into a 2-stage shared-memory ring in the 128-byte-swizzled UMMA
//                        layout: the int8 state prefix is dequantised there exactly as materialize() rounds
//                        (bf16(q * s); fp16 scales: bf16(fp16(q * s))), the bf16 question prefix and own keys are
//                        copied; a per-key bias marks padding / holes
//   MMA warp (1 thread)  S_{j+1} = Q K_{j+1}^T into the other half of a double-buffered S in TMEM while the softmax
//                        works on S_j, then O += P_j V_j (V as an MN-major operand) with O in TMEM
//   softmax warps (4)    read the slot's S row from TMEM, mask (causal and same-row for own keys), online softmax in
//                        the exp2 domain with a lazy rescale of O only when the max grows by more than 2^8, P (bf16)
//                        into a double-buffered shared-memory tile; at the end O / l and the natural-log LSE
// Every mbarrier wait is bounded; a time-out ends the kernel with an error code, never a hang.
// Each slot's math does not depend on the other slots: outputs do not depend on row order.
#include <cudaTypedefs.h>

#include <string.h>

#include <type_traits>

#include "sm100.cuh"

namespace od {
namespace {
using namespace sm100;

constexpr int kSoftmaxWarps = 4;     // warps 0-3: thread = query slot = TMEM lane
constexpr int kMmaWarp = 4;          // warp 4: TMEM allocation and the single MMA-issuing thread
constexpr int kProducerWarps = 4;    // warps 5-8: stage K/V blocks
constexpr int kProducers = 32 * kProducerWarps;
constexpr int kThreads = 32 * (kSoftmaxWarps + 1 + kProducerWarps);
constexpr int BM = 128;              // query slots per CTA
constexpr int BN = 64;               // keys per block
constexpr int kStages = 3;           // K/V ring depth
constexpr uint32_t kTmemCols = 256;  // S buffers at columns 0 and 64 (64 fp32 each), O at column 128 (D fp32)
constexpr uint32_t kTmemO = 128;
constexpr int32_t kErrAttn = 0x5A0000;

template <int D>
struct Layout {
  static constexpr int Q = 0;                        // BM x D bf16: D/64 atoms of BM rows x 128 B
  static constexpr int Q_ATOM = BM * 128;
  static constexpr int KV_ATOM = BN * 128;           // a K or V block: D/64 atoms of BN rows x 128 B
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int KV0 = Q + BM * D * 2;         // stage b: K at KV0 + 2b*KV_BYTES, V right after
  static constexpr int P0 = KV0 + 2 * kStages * KV_BYTES;  // P buffer b: BM x BN bf16 (one atom)
  static constexpr int BIAS0 = P0 + 2 * BM * BN * 2; // bias of stage b: BN floats at BIAS0 + b*BN*4
  static constexpr int BAR = BIAS0 + kStages * BN * 4;  // mbarriers + TMEM holder + abort flag
  static constexpr int BYTES = BAR + 128 + 1024;     // + alignment slack
  static __host__ __device__ constexpr int K(int b) { return KV0 + 2 * b * KV_BYTES; }
  static __host__ __device__ constexpr int V(int b) { return KV0 + (2 * b + 1) * KV_BYTES; }
  static __host__ __device__ constexpr int P(int b) { return P0 + b * BM * BN * 2; }
  static __host__ __device__ constexpr int BIAS(int b) { return BIAS0 + b * BN * 4; }
};

struct Params {
  CUtensorMap map_ko, map_vo, map_kq, map_vq;   // bf16 (rows, Hkv*D) views of own / question K and V, 64x64 boxes
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
  const int32_t* row_groups;
  __nv_bfloat16* o;
  float* lse;
  int32_t* err;
  int64_t t, T, Lq;
  int Hq, Hkv, rep, tiles_per_group;
  float scale_log2;
};

// byte offset of 16-byte chunk `ch` of row `row` in a 128B-swizzled tile made of `atom`-byte column atoms
__device__ __forceinline__ uint32_t swz(int row, int ch, int atom) {
  return static_cast<uint32_t>((ch >> 3) * atom + row * 128 + (((ch & 7) ^ (row & 7)) << 4));
}

// 2^x by the hardware approximation (ex2.approx; relative error ~2^-22, exact 0 for -inf): the softmax weights
// are rounded to bf16 before P.V anyway.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One producer thread's share of an int8 K/V block held in registers between its load and its dequantising store,
// so the next blocks' loads are in flight while this one is converted.
template <int D>
struct RawInt8 {
  static constexpr int N = BN * (D / 16) / kProducers;   // 16-byte chunks per thread per matrix
  int4 k[N], v[N];
  float ks[N], vs[N];
};

template <typename TS, int D>
__device__ __forceinline__ void load_int8(RawInt8<D>& r, int pt, const int8_t* Kb, const int8_t* Vb, const TS* ks,
                                          const TS* vs, int p0, int p_hi) {
  constexpr int CPR = D / 16;
#pragma unroll
  for (int it = 0; it < RawInt8<D>::N; ++it) {
    const int c = pt + it * kProducers;
    const int key = c / CPR, ch = c % CPR;
    const int p = p0 + key;
    if (p < p_hi) {
      r.k[it] = __ldg(reinterpret_cast<const int4*>(Kb + static_cast<int64_t>(p) * D) + ch);
      r.v[it] = __ldg(reinterpret_cast<const int4*>(Vb + static_cast<int64_t>(p) * D) + ch);
      r.ks[it] = Elem<TS>::to_f(ks[p]);
      r.vs[it] = Elem<TS>::to_f(vs[p]);
    } else {
      r.k[it] = r.v[it] = make_int4(0, 0, 0, 0);
      r.ks[it] = r.vs[it] = 0.f;
    }
  }
}

// Dequantise a held block into the stage exactly as materialize() rounds; keys >= p_hi or masked by pmask get
// bias -inf (their data is zero).
template <typename TS, int D>
__device__ __forceinline__ void store_int8(const RawInt8<D>& r, uint8_t* sK, uint8_t* sV, float* bias, int pt,
                                           const uint8_t* pm, int p0, int p_hi) {
  using L = Layout<D>;
  constexpr int CPR = D / 16;
#pragma unroll
  for (int it = 0; it < RawInt8<D>::N; ++it) {
    const int c = pt + it * kProducers;
    const int key = c / CPR, ch = c % CPR;
    const int p = p0 + key;
    const int8_t* kb = reinterpret_cast<const int8_t*>(&r.k[it]);
    const int8_t* vb = reinterpret_cast<const int8_t*>(&r.v[it]);
    uint32_t kw[8], vw[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float k0 = static_cast<float>(kb[2 * e]) * r.ks[it], k1 = static_cast<float>(kb[2 * e + 1]) * r.ks[it];
      float v0 = static_cast<float>(vb[2 * e]) * r.vs[it], v1 = static_cast<float>(vb[2 * e + 1]) * r.vs[it];
      if (std::is_same<TS, __half>::value) {
        k0 = rhf(k0); k1 = rhf(k1); v0 = rhf(v0); v1 = rhf(v1);
      }
      kw[e] = pack_bf16(k0, k1);
      vw[e] = pack_bf16(v0, v1);
    }
    // the 16 int8 values of chunk ch are bf16 chunks 2ch and 2ch+1 of the row
    *reinterpret_cast<uint4*>(sK + swz(key, 2 * ch, L::KV_ATOM)) = make_uint4(kw[0], kw[1], kw[2], kw[3]);
    *reinterpret_cast<uint4*>(sK + swz(key, 2 * ch + 1, L::KV_ATOM)) = make_uint4(kw[4], kw[5], kw[6], kw[7]);
    *reinterpret_cast<uint4*>(sV + swz(key, 2 * ch, L::KV_ATOM)) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
    *reinterpret_cast<uint4*>(sV + swz(key, 2 * ch + 1, L::KV_ATOM)) = make_uint4(vw[4], vw[5], vw[6], vw[7]);
    if (ch == 0) bias[key] = (p < p_hi && (!pm || pm[p])) ? 0.f : -INFINITY;
  }
}

// Warp-uniform bounded wait (the softmax warps issue warp-collective TMEM loads after it).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int32_t* err,
                                          int32_t code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, err, code));
}

template <typename TS, int D>
__global__ void __launch_bounds__(kThreads, 1) prefix_attn_kernel(const __grid_constant__ Params P) {
  using L = Layout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // pointer arithmetic on the shared array (not an integer cast) keeps the shared address space visible to the
  // compiler, so accesses compile to shared-memory instructions rather than generic ones
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* kv_full = bars;                    // [kStages] producers -> MMA / softmax (count 128)
  uint64_t* kv_empty = bars + kStages;         // [kStages] MMA (after PV_j) -> producers
  uint64_t* s_full = bars + 2 * kStages;       // [2] MMA (after S_j) -> softmax
  uint64_t* p_full = s_full + 2;               // [2] softmax (P_j written) -> MMA (count 128)
  uint64_t* pv_done = s_full + 4;              // [2] MMA (after PV_j) -> softmax
  uint64_t* drain = s_full + 6;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % P.tiles_per_group;
  const int grp = blockIdx.x / P.tiles_per_group;
  const int row0 = P.row_groups ? P.row_groups[2 * grp] : grp;
  const int nr = P.row_groups ? P.row_groups[2 * grp + 1] : 1;
  const int g = blockIdx.y, rep = P.rep;
  const int t = static_cast<int>(P.t);
  const int slots_row = t * rep;
  const int slots = nr * slots_row;
  const int s0 = tile * BM;
  if (s0 >= slots) return;                            // uniform: before any barrier or allocation

  if (tid == 0) {
    for (int b = 0; b < kStages; ++b) {
      mbar_init(&kv_full[b], kProducers);
      mbar_init(&kv_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 32 * kSoftmaxWarps);
      mbar_init(&pv_done[b], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_holder, kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // ---- key segments (the group's rows share their state and question); every role derives the same schedule
  int nb1 = 0, lo1 = 0, hi1 = 0, st = 0;
  if (P.Kp) {
    st = P.row_state[row0];
    lo1 = P.p_lo ? P.p_lo[st] : 0;
    hi1 = P.p_hi ? P.p_hi[st] : static_cast<int>(P.T);
    nb1 = hi1 > lo1 ? (hi1 - lo1 + BN - 1) / BN : 0;
  }
  int nb2 = 0, n2 = 0, qr = 0;
  if (P.Kq) {
    qr = P.row_q[row0];
    n2 = P.q_len[qr];
    nb2 = (n2 + BN - 1) / BN;
  }
  // own keys, flattened (row a, token j) -> a * t + j; a single long row only needs keys up to the tile's last token
  int own_begin = 0, own_end = nr * t;
  if (nr == 1) {
    const int lo = P.own_lo ? P.own_lo[row0] : 0;
    const int last_tok = min(t - 1, (min(slots, s0 + BM) - 1) / rep);
    own_begin = (lo / BN) * BN;
    own_end = last_tok + 1;
  }
  const int nb3 = own_end > own_begin ? (own_end - own_begin + BN - 1) / BN : 0;
  const int nblk = nb1 + nb2 + nb3;

  if (warp >= kSoftmaxWarps + 1) {
    // ================================================================== producers: Q, then K/V blocks
    const int pt = tid - 32 * (kSoftmaxWarps + 1);
    {
      constexpr int CPR = D / 8;
#pragma unroll 4
      for (int c = pt; c < BM * CPR; c += kProducers) {
        const int r = c / CPR, ch = c % CPR;
        const int s = s0 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (s < slots) {
          const int a = s / slots_row, i = (s % slots_row) / rep, hh = s % rep;
          v = __ldg(reinterpret_cast<const uint4*>(
                        P.q + ((static_cast<int64_t>(row0 + a) * t + i) * P.Hq + g * rep + hh) * D) + ch);
        }
        *reinterpret_cast<uint4*>(sm + L::Q + swz(r, ch, L::Q_ATOM)) = v;
      }
    }
    const int8_t* Kb1 = nullptr;
    const int8_t* Vb1 = nullptr;
    const TS* ks1 = nullptr;
    const TS* vs1 = nullptr;
    const uint8_t* pm1 = nullptr;
    if (P.Kp) {
      const int64_t base = (static_cast<int64_t>(st) * P.Hkv + g) * P.T;
      Kb1 = P.Kp + base * D;
      Vb1 = P.Vp + base * D;
      ks1 = static_cast<const TS*>(P.ksc) + base;
      vs1 = static_cast<const TS*>(P.vsc) + base;
      pm1 = P.pmask ? P.pmask + static_cast<int64_t>(st) * P.T : nullptr;
    }
    // int8 blocks run a 2-deep register pipeline: blocks j+1 and j+2 are being loaded while block j is converted
    RawInt8<D> ra, rb;
    if (nb1 > 0) load_int8<TS, D>(ra, pt, Kb1, Vb1, ks1, vs1, lo1, hi1);
    if (nb1 > 1) load_int8<TS, D>(rb, pt, Kb1, Vb1, ks1, vs1, lo1 + BN, hi1);
    for (int j = 0; j < nblk; ++j) {
      const int b = j % kStages;
      if (j >= kStages && !mbar_wait(&kv_empty[b], ((j / kStages) - 1) & 1, abort_flag, P.err, kErrAttn | 1)) break;
      uint8_t* sK = sm + L::K(b);
      uint8_t* sV = sm + L::V(b);
      float* bias = reinterpret_cast<float*>(sm + L::BIAS(b));
      if (j < nb1) {
        store_int8<TS, D>(ra, sK, sV, bias, pt, pm1, lo1 + j * BN, hi1);
        ra = rb;
        if (j + 2 < nb1) load_int8<TS, D>(rb, pt, Kb1, Vb1, ks1, vs1, lo1 + (j + 2) * BN, hi1);
      } else {
        // bf16 block: TMA straight into the swizzled UMMA layout; every producer thread writes a key's bias first
        const bool q_seg = j < nb1 + nb2;
        const int k0 = q_seg ? (j - nb1) * BN : own_begin + (j - nb1 - nb2) * BN;
        if (pt < BN) {
          const int idx = k0 + pt;
          bool ok;
          if (q_seg) {
            ok = idx < n2;
          } else {
            const int a = idx / t, jj = idx - a * t;
            const int r = row0 + a;
            ok = idx < own_end && a < nr && jj >= (P.own_lo ? P.own_lo[r] : 0) && jj < (P.own_hi ? P.own_hi[r] : t);
          }
          bias[pt] = ok ? 0.f : -INFINITY;
        }
        if (pt == 0) {
          const CUtensorMap* mk = q_seg ? &P.map_kq : &P.map_ko;
          const CUtensorMap* mv = q_seg ? &P.map_vq : &P.map_vo;
          const int y = (q_seg ? qr * static_cast<int>(P.Lq) : row0 * t) + k0;
          mbar_arrive_expect_tx(&kv_full[b], 2 * L::KV_BYTES);
#pragma unroll
          for (int h = 0; h < D / 64; ++h) {
            tma_load_2d(sK + h * L::KV_ATOM, mk, &kv_full[b], g * D + h * 64, y);
            tma_load_2d(sV + h * L::KV_ATOM, mv, &kv_full[b], g * D + h * 64, y);
          }
        } else {
          mbar_arrive(&kv_full[b]);
        }
        continue;
      }
      fence_proxy_async_smem();
      mbar_arrive(&kv_full[b]);
    }
  } else if (warp == kMmaWarp) {
    // ================================================================== MMA issue (one thread)
    if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(BM, BN, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BM, D, true);
      const uint32_t sQ = smem_u32(sm + L::Q);
      auto issue_s = [&](int j) {
        const int b = j & 1;
        const uint32_t sK = smem_u32(sm + L::K(j % kStages));
#pragma unroll
        for (int kd = 0; kd < D / 16; ++kd) {
          const uint32_t qa = sQ + (kd >> 2) * L::Q_ATOM + (kd & 3) * 32;
          const uint32_t ka = sK + (kd >> 2) * L::KV_ATOM + (kd & 3) * 32;
          mma_f16(tmem + b * BN, desc_sw128(qa, 16, 1024), desc_sw128(ka, 16, 1024), idesc_qk, kd > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[b]);
      };
      bool live = mbar_wait(&kv_full[0], 0, abort_flag, P.err, kErrAttn | 2);
      if (live) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; j < nblk && live; ++j) {
        if (j + 1 < nblk) {
          const int b1 = (j + 1) % kStages;
          if (!mbar_wait(&kv_full[b1], ((j + 1) / kStages) & 1, abort_flag, P.err, kErrAttn | 3)) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        const int b = j & 1;
        if (!mbar_wait(&p_full[b], (j >> 1) & 1, abort_flag, P.err, kErrAttn | 4)) break;
        tc_fence_after();
        const uint32_t sP = smem_u32(sm + L::P(b)), sV = smem_u32(sm + L::V(j % kStages));
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)
          mma_f16(tmem + kTmemO, desc_sw128(sP + kk * 32, 16, 1024),
                  desc_sw128(sV + kk * 16 * 128, L::KV_ATOM, 1024), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&kv_empty[j % kStages]);
        mma_commit(&pv_done[b]);
      }
      // every MMA issued here has completed before TMEM is released (immediate unless aborted)
      mma_commit(drain);
      const long long c0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - c0 < kWaitLimitCycles) {
      }
    }
  } else {
    // ================================================================== softmax (thread = slot = TMEM lane)
    const int slot = s0 + tid;
    const bool my_valid = slot < slots;
    const int a_my = my_valid ? slot / slots_row : 0;
    const int i_my = my_valid ? (slot % slots_row) / rep : 0;
    const int hh_my = slot % rep;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float m_used = -INFINITY, l_sum = 0.f;
    bool live = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!warp_wait(&s_full[b], ph, abort_flag, P.err, kErrAttn | 5) ||
          !warp_wait(&kv_full[j % kStages], (j / kStages) & 1, abort_flag, P.err, kErrAttn | 6)) {
        live = false;
        break;
      }
      tc_fence_after();
      float s[BN];
      {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tmem + lane_off + b * BN, r0);
        tmem_ld_32x32b_x32(tmem + lane_off + b * BN + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          s[k] = __uint_as_float(r0[k]);
          s[k + 32] = __uint_as_float(r1[k]);
        }
      }
      float bias[BN];
      {
        const float4* bsrc = reinterpret_cast<const float4*>(sm + L::BIAS(j % kStages));
#pragma unroll
        for (int k = 0; k < BN / 4; ++k) {
          const float4 b4 = bsrc[k];
          bias[4 * k] = b4.x;
          bias[4 * k + 1] = b4.y;
          bias[4 * k + 2] = b4.z;
          bias[4 * k + 3] = b4.w;
        }
      }
      const bool own = j >= nb1 + nb2;
      const float scale = P.scale_log2;
      float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (!own) {
#pragma unroll
        for (int k = 0; k < BN; ++k) {
          s[k] = fmaf(s[k], scale, bias[k]);
          mq[k & 3] = fmaxf(mq[k & 3], s[k]);
        }
      } else {
        // own keys visible to this slot form one range of the flattened (row, token) index: its own row's tokens
        // up to its own position (padding inside the row is already in the bias)
        const int key0 = own_begin + (j - nb1 - nb2) * BN;
        const int vis_lo = a_my * t - key0, vis_hi = a_my * t + i_my - key0;
#pragma unroll
        for (int k = 0; k < BN; ++k) {
          s[k] = (k < vis_lo || k > vis_hi) ? -INFINITY : fmaf(s[k], scale, bias[k]);
          mq[k & 3] = fmaxf(mq[k & 3], s[k]);
        }
      }
      const float mb = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      float alpha = 1.f;
      bool resc = false;
      if (m_used == -INFINITY) {
        m_used = mb;                                   // nothing accumulated yet: O and l are 0
      } else if (mb > m_used + 8.f) {
        alpha = ex2_approx(m_used - mb);
        l_sum *= alpha;
        m_used = mb;
        resc = true;
      }
      uint32_t pw[BN / 2];
      float rq[4] = {0.f, 0.f, 0.f, 0.f};
      if (m_used == -INFINITY) {                       // no visible key so far: every weight is 0
#pragma unroll
        for (int k = 0; k < BN / 2; ++k) pw[k] = 0u;
      } else {
#pragma unroll
        for (int k = 0; k < BN; k += 2) {
          const float p0 = ex2_approx(s[k] - m_used);
          const float p1 = ex2_approx(s[k + 1] - m_used);
          rq[(k >> 1) & 3] += p0 + p1;
          pw[k / 2] = pack_bf16(p0, p1);
        }
      }
      const float rs = (rq[0] + rq[1]) + (rq[2] + rq[3]);
      l_sum += rs;
      // P buffer b is free once PV_{j-2} completed
      if (j >= 2 && !warp_wait(&pv_done[b], ((j >> 1) - 1) & 1, abort_flag, P.err, kErrAttn | 7)) {
        live = false;
        break;
      }
      if (__any_sync(0xffffffffu, resc)) {           // lazy rescale of this warp's O rows once PV_{j-1} is done
        if (!warp_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, P.err, kErrAttn | 8)) {
          live = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + lane_off + kTmemO + dc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
          tmem_st_32x32b_x32(tmem + lane_off + kTmemO + dc * 32, o);
        }
        tmem_st_wait();
      }
      uint8_t* sP = sm + L::P(b);
#pragma unroll
      for (int c = 0; c < BN / 8; ++c)
        *reinterpret_cast<uint4*>(sP + swz(tid, c, BM * 128)) =
            make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
    }
    // ---- epilogue: O / l, natural-log LSE (nothing is written after a time-out; the error word says why).
    // TMEM loads are warp-collective: every lane loads, valid slots store.
    if (live && nblk > 0)
      live = warp_wait(&pv_done[(nblk - 1) & 1], ((nblk - 1) >> 1) & 1, abort_flag, P.err, kErrAttn | 9);
    if (live) {
      tc_fence_after();
      const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
      const int64_t orow = ((static_cast<int64_t>(row0 + a_my) * t + i_my) * P.Hq + g * rep + hh_my) * D;
#pragma unroll 1
      for (int dc = 0; dc < D / 32; ++dc) {
        uint32_t o[32];
        if (nblk > 0) {
          tmem_ld_32x32b_x32(tmem + lane_off + kTmemO + dc * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = 0u;
        }
        if (my_valid) {
          uint32_t w[16];
#pragma unroll
          for (int k = 0; k < 16; ++k)
            w[k] = pack_bf16(__uint_as_float(o[2 * k]) * inv, __uint_as_float(o[2 * k + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(P.o + orow + dc * 32);
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
        }
      }
      if (P.lse && my_valid)
        P.lse[(static_cast<int64_t>(row0 + a_my) * P.Hq + g * rep + hh_my) * t + i_my] =
            l_sum > 0.f ? (m_used + log2f(l_sum)) * 0.6931471805599453f : -INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// (rows, cols) bf16 row-major view tiled into 64 x 64 boxes with the 128-byte swizzle of the UMMA layout
int make_map_bf16(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BN)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled (bf16) failed (%d)", static_cast<int>(r));
  return OD_OK;
}

template <typename TS, int D>
int launch_attn(const Params& P, dim3 grid, cudaStream_t st) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(prefix_attn_kernel<TS, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Layout<D>::BYTES));
    attr[dev] = true;
  }
  prefix_attn_kernel<TS, D><<<grid, kThreads, Layout<D>::BYTES, st>>>(P);
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
                              const int32_t* row_groups, void* o, float* lse, od_attn_dims dims, void* stream) {
  OD_REQUIRE(q && k_own && v_own && o, "od_prefix_attn: null pointer");
  OD_REQUIRE(dims.D == 64 || dims.D == 128, "od_prefix_attn: head_dim %d not in {64, 128}", dims.D);
  OD_REQUIRE(dims.Hq > 0 && dims.Hkv > 0 && dims.Hq % dims.Hkv == 0, "od_prefix_attn: bad head counts");
  const int rep = dims.Hq / dims.Hkv;
  OD_REQUIRE(dims.R >= 0 && dims.t >= 0 && dims.t < (1 << 24), "od_prefix_attn: bad R/t");
  OD_REQUIRE(!Kp || (Vp && ksc && vsc && row_state && dims.S > 0 && dims.T > 0 && dims.T < (1 << 30)),
             "od_prefix_attn: the int8 prefix needs Vp, scales, row_state, S, T");
  OD_REQUIRE(!Kp || dims.scale_dtype == OD_BF16 || dims.scale_dtype == OD_F16, "od_prefix_attn: scale dtype");
  OD_REQUIRE(!Kq || (Vq && row_q && q_len && dims.NQ > 0 && dims.Lq > 0), "od_prefix_attn: bad question prefix");
  OD_REQUIRE(aligned16(q) && aligned16(k_own) && aligned16(v_own) && aligned16(o) &&
                 (!Kp || (aligned16(Kp) && aligned16(Vp))) && (!Kq || (aligned16(Kq) && aligned16(Vq))),
             "od_prefix_attn: tensors must be 16-byte aligned");
  const int64_t G = row_groups ? dims.G : dims.R;
  const int64_t max_rows = row_groups ? dims.max_group_rows : 1;
  OD_REQUIRE(G >= 0 && max_rows >= 1, "od_prefix_attn: bad row groups");
  OD_REQUIRE(max_rows == 1 || max_rows * dims.t * rep <= BM,
             "od_prefix_attn: a group of several rows must fit one %d-slot tile (rows %lld x t %lld x rep %d)", BM,
             (long long)max_rows, (long long)dims.t, rep);
  if (G == 0 || dims.t == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_prefix_attn: no device error word");
  Params P;
  memset(&P, 0, sizeof(P));
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
  P.row_groups = row_groups;
  P.o = static_cast<__nv_bfloat16*>(o);
  P.lse = lse;
  P.err = err;
  P.t = dims.t;
  P.T = dims.T;
  P.Lq = dims.Lq;
  P.Hq = dims.Hq;
  P.Hkv = dims.Hkv;
  P.rep = rep;
  P.tiles_per_group = static_cast<int>((max_rows * dims.t * rep + BM - 1) / BM);
  P.scale_log2 = dims.sm_scale * 1.4426950408889634f;
  {
    const uint64_t cols = static_cast<uint64_t>(dims.Hkv) * dims.D;
    OD_REQUIRE((cols * 2) % 16 == 0, "od_prefix_attn: Hkv * D * 2 must be a multiple of 16");
    int rc = make_map_bf16(&P.map_ko, k_own, cols, static_cast<uint64_t>(dims.R * dims.t));
    if (!rc) rc = make_map_bf16(&P.map_vo, v_own, cols, static_cast<uint64_t>(dims.R * dims.t));
    if (!rc && Kq) rc = make_map_bf16(&P.map_kq, Kq, cols, static_cast<uint64_t>(dims.NQ * dims.Lq));
    if (!rc && Kq) rc = make_map_bf16(&P.map_vq, Vq, cols, static_cast<uint64_t>(dims.NQ * dims.Lq));
    if (!Kq) {
      P.map_kq = P.map_ko;
      P.map_vq = P.map_vo;
    }
    if (rc) return rc;
  }
  const int64_t gx = G * P.tiles_per_group;
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
