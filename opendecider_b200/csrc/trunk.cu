// The V3 decision trunk in fp32 on sm_100a (reference src/opendecider/v3.py: ScaleNorm :43-50, XATGLU :53-67,
// rope :70-79, MHA :82-100, V3.forward :606-709, the layer mix V3._mix_wide :328-341):
//   gemm_f32_kernel        y = x W^T (+ bias) (+ residual), fp32 in and out, on the tensor cores as three tf32
//                          products per k-step (x_hi W_hi + x_hi W_lo + x_lo W_hi, "3xTF32"): every fp32 operand is
//                          held as hi = x rounded to tf32 plus lo = x - hi (exact), so the products carry ~22 bits of
//                          each operand and the fp32 TMEM accumulator gives fp32-level results (the lo x lo term,
//                          2^-22 relative, is left out). 128 x 128 tiles, K in 32-element (128-byte) steps through a
//                          3-stage TMA ring of the four operand halves, two TMEM accumulators, persistent CTAs.
//                          The epilogue adds the bias and the residual (x = x + layer(x) in place, or a broadcast
//                          row), can scatter rows to given output rows (the padded option/context layouts) and
//                          applies RoPE to the q / k columns of an attention's projection as it writes them.
//   scalenorm_split_kernel ScaleNorm g * x / max(||x||, eps) of each row - of the softmax-weighted mix of the feature
//                          layers first for the input projections - written as the hi / lo operand pair
//   xatglu_split_kernel    the first-order xATGLU gate ((atan z + pi/2) / pi)(1 + 2a) - a times the value
//                          projection, written as the hi / lo operand pair of the output projection
//   trunk_attn_kernel      softmax(q k^T / sqrt(dh) + bias) v per (question, head) with the trunk's masks built from
//                          group ids instead of an (N, h, P, T) bias tensor: same-option bonus + key padding (the
//                          self-attention over option tokens), key padding (the cross-attention to the question),
//                          keys of the query's own option only (the CLS readout); a SIMT flash attention in fp32
//                          with 4 x 4 register tiles, K / V streamed through shared memory by cp.async
// Every wait of the GEMM is bounded: a time-out records an error code in the device error word and ends the kernel.
#include <cudaTypedefs.h>
#include <math.h>

#include "sm100.cuh"

namespace od {
namespace {
using namespace sm100;

constexpr int32_t kErrTrunk = 0x540000;

// x rounded to the nearest tf32 (10 explicit mantissa bits; ties away from zero) and the exact remainder
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
  lo = __fsub_rn(x, hi);
}

// ---------------------------------------------------------------------------------------------- fp32 GEMM (3xTF32)
constexpr int FB = 128;                          // tile rows of x and of W
constexpr int FK = 32;                           // fp32 elements of one 128-byte swizzle row: K per stage
constexpr int F_STAGES = 3;
constexpr int F_OPER = FB * FK * 4;              // 16 KB: one half (hi or lo) of the x or the W tile
constexpr int F_STAGE = 4 * F_OPER;              // x hi, x lo, W hi, W lo
constexpr int kFThreads = 192;                   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kFTmemCols = 2 * FB;
constexpr int kFSmem = F_STAGES * F_STAGE + 1024 /*barriers*/ + 1024 /*alignment slack*/;

struct GemmF32Args {
  float* y;
  int64_t ldy;
  const float* bias;         // (N,) or null
  const float* res;          // residual rows (row r at res + out_row(r) * ldres; ldres 0 = one broadcast row) or null
  int64_t ldres;
  const int64_t* out_rows;   // (M,) output row of each x row, or null (identity)
  const int32_t* rope_pos;   // (M,) RoPE position of each x row, or null
  const float* rope_inv;     // (rope_dh / 2,) the rotation frequencies 1 / 10000^(2i / rope_dh)
  int rope_cols, rope_dh;    // columns [0, rope_cols) rotated in pairs (2i, 2i+1) of rope_dh-wide heads
  int M, N, K;
  int vec;                   // y / res rows allow 16-byte accesses
};

__global__ void __launch_bounds__(kFThreads, 1)
    gemm_f32_kernel(const __grid_constant__ CUtensorMap tXh, const __grid_constant__ CUtensorMap tXl,
                    const __grid_constant__ CUtensorMap tWh, const __grid_constant__ CUtensorMap tWl,
                    const GemmF32Args a, int32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + F_STAGES * F_STAGE);
  uint64_t* empty = full + F_STAGES;
  uint64_t* tfull = empty + F_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  __shared__ float rope_inv[64];                     // the RoPE epilogue's frequencies
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_n = (a.N + FB - 1) / FB, num_kb = (a.K + FK - 1) / FK;
  const int num_tiles = ((a.M + FB - 1) / FB) * num_n;
  if (a.rope_pos && static_cast<int>(threadIdx.x) < a.rope_dh / 2) rope_inv[threadIdx.x] = a.rope_inv[threadIdx.x];

  if (threadIdx.x == 0) {
    for (int s = 0; s < F_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tXh);
    tma_prefetch_desc(&tXl);
    tma_prefetch_desc(&tWh);
    tma_prefetch_desc(&tWl);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kFTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, armed = 0, armed_par = 0;
      bool live = true;
      for (int tile = blockIdx.x; tile < num_tiles && live; tile += gridDim.x) {
        const int m0 = (tile / num_n) * FB, n0 = (tile % num_n) * FB;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrTrunk | 1)) {
            live = false;
            break;
          }
          uint8_t* st_ = smem + stage * F_STAGE;
          mbar_arrive_expect_tx(&full[stage], F_STAGE);
          tma_load_2d(st_, &tXh, &full[stage], kb * FK, m0);
          tma_load_2d(st_ + F_OPER, &tXl, &full[stage], kb * FK, m0);
          tma_load_2d(st_ + 2 * F_OPER, &tWh, &full[stage], kb * FK, n0);
          tma_load_2d(st_ + 3 * F_OPER, &tWl, &full[stage], kb * FK, n0);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          if (++stage == F_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!live) {   // aborted: let the loads already issued land before shared memory goes away (bounded)
        for (int s = 0; s < F_STAGES; ++s)
          if (armed & (1u << s)) {
            const long long c0 = clock64();
            while (!mbar_try_wait(&full[s], (armed_par >> s) & 1) && clock64() - c0 < kWaitLimitCycles) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(FB, FB);
      int stage = 0;
      uint32_t phase = 0;
      bool live = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && live; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1, abort_flag, err, kErrTrunk | 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * FB;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, err, kErrTrunk | 3)) {
            live = false;
            break;
          }
          tc_fence_after();
          const uint32_t xh = smem_u32(smem + stage * F_STAGE);
          const uint32_t xl = xh + F_OPER, wh = xh + 2 * F_OPER, wl = xh + 3 * F_OPER;
#pragma unroll
          for (int k = 0; k < FK / 8; ++k) {            // 8 tf32 = 32 bytes of each row per MMA
            mma_tf32(d_tmem, desc_kmajor_sw128(xh + 32 * k), desc_kmajor_sw128(wl + 32 * k), idesc, (kb | k) != 0);
            mma_tf32(d_tmem, desc_kmajor_sw128(xl + 32 * k), desc_kmajor_sw128(wh + 32 * k), idesc, 1);
            mma_tf32(d_tmem, desc_kmajor_sw128(xh + 32 * k), desc_kmajor_sw128(wh + 32 * k), idesc, 1);
          }
          mma_commit(&empty[stage]);
          if (++stage == F_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (live) mma_commit(&tfull[acc]);
      }
      mma_commit(drain);      // every MMA issued here has completed before TMEM is released
      const long long c0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - c0 < kWaitLimitCycles) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue: one row per thread
    const int quarter = warp & 3;                    // TMEM lanes 32 * quarter .. + 31 = tile rows
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      if (!mbar_wait(&tfull[acc], (local >> 1) & 1, abort_flag, err, kErrTrunk | 4)) break;
      tc_fence_after();
      const int m0 = (tile / num_n) * FB, n0 = (tile % num_n) * FB;
      const int row = m0 + quarter * 32 + lane;
      const int64_t orow = row < a.M ? (a.out_rows ? a.out_rows[row] : row) : -1;
      const float rpos = a.rope_pos && row < a.M ? static_cast<float>(a.rope_pos[row]) : 0.f;
      const uint32_t tb = tmem_base + acc * FB + (static_cast<uint32_t>(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < FB / 32; ++c) {
        const int col0 = n0 + c * 32;
        if (col0 >= a.N) break;                      // uniform across the warp
        uint32_t r[32];
        tmem_ld_32x32b_x32(tb + c * 32, r);
        tmem_ld_wait();
        if (orow < 0) continue;
        float* yr = a.y + orow * a.ldy;
        const float* rr = a.res ? a.res + orow * a.ldres : nullptr;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const int col = col0 + j;
          if (col < a.N) {
            float v[4] = {__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                          __uint_as_float(r[j + 3])};
            const bool full4 = a.vec && col + 3 < a.N;
            if (a.bias) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (col + i < a.N) v[i] = __fadd_rn(v[i], __ldg(a.bias + col + i));
            }
            if (a.rope_pos && col < a.rope_cols) {   // RoPE (v3.py:70-79) of the pairs (col, col+1), (col+2, col+3)
#pragma unroll
              for (int i = 0; i < 4; i += 2) {
                const float ang = __fmul_rn(rpos, rope_inv[((col + i) % a.rope_dh) >> 1]);
                const float cs = cosf(ang), sn = sinf(ang);
                const float x1 = v[i], x2 = v[i + 1];
                v[i] = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
                v[i + 1] = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
              }
            }
            if (rr) {
              if (full4) {
                const float4 q = *reinterpret_cast<const float4*>(rr + col);
                v[0] = __fadd_rn(q.x, v[0]);
                v[1] = __fadd_rn(q.y, v[1]);
                v[2] = __fadd_rn(q.z, v[2]);
                v[3] = __fadd_rn(q.w, v[3]);
              } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  if (col + i < a.N) v[i] = __fadd_rn(rr[col + i], v[i]);
              }
            }
            if (full4) {
              *reinterpret_cast<float4*>(yr + col) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (col + i < a.N) yr[col + i] = v[i];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kFTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------- split / ScaleNorm
__global__ void split_tf32_kernel(const float* __restrict__ x, int64_t ldx, int64_t M, int64_t K,
                                  float* __restrict__ hi, float* __restrict__ lo, int64_t ldo) {
  const int64_t n = M * K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / K, c = i - r * K;
    float h, l;
    split_tf32(x[r * ldx + c], h, l);
    hi[r * ldo + c] = h;
    lo[r * ldo + c] = l;
  }
}

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) { return Elem<T>::to_f(*p); }

constexpr int kNormThreads = 128;

// One CTA per row; VPT elements per thread held in registers (K <= 128 * VPT).
template <typename T, int VPT>
__global__ void __launch_bounds__(kNormThreads) scalenorm_split_kernel(const T* __restrict__ x, int64_t ldx, int K,
                                                                       const float* __restrict__ mixw, int n_mix,
                                                                       const float* __restrict__ g, float eps,
                                                                       float* __restrict__ hi, float* __restrict__ lo,
                                                                       int64_t ldo) {
  __shared__ float red[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  float v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = j * kNormThreads + threadIdx.x;
    float s = 0.f;
    if (e < K) {
      if (mixw) {       // sum over the feature layers of w_l * f_l (layer l at columns l * K ..)
        s = __fmul_rn(__ldg(mixw), ld_f(xr + e));
        for (int l = 1; l < n_mix; ++l) s = fmaf(__ldg(mixw + l), ld_f(xr + static_cast<int64_t>(l) * K + e), s);
      } else {
        s = ld_f(xr + e);
      }
    }
    v[j] = s;
    ss = fmaf(s, s, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float d = fmaxf(__fsqrt_rn(tot), eps);
  const float gg = __ldg(g);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = j * kNormThreads + threadIdx.x;
    if (e < K) {
      float h, l;
      split_tf32(__fdiv_rn(__fmul_rn(gg, v[j]), d), h, l);
      hi[row * ldo + e] = h;
      lo[row * ldo + e] = l;
    }
  }
}

// ((atan z + pi/2) / pi)(1 + 2a) - a, times the value projection; z = zv[:, :F], value = zv[:, F:2F]
__global__ void xatglu_split_kernel(const float* __restrict__ zv, int64_t ldzv, int64_t M, int64_t F,
                                    const float* __restrict__ alpha, float* __restrict__ hi, float* __restrict__ lo,
                                    int64_t ldo) {
  const float a = __ldg(alpha);
  const float amp = __fadd_rn(1.0f, __fmul_rn(2.0f, a));
  constexpr float kHalfPi = 1.57079632679489662f, kPi = 3.14159265358979323f;
  const int64_t n = M * F;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / F, c = i - r * F;
    const float z = zv[r * ldzv + c], val = zv[r * ldzv + F + c];
    const float gate = __fsub_rn(__fmul_rn(__fdiv_rn(__fadd_rn(atanf(z), kHalfPi), kPi), amp), a);
    float h, l;
    split_tf32(__fmul_rn(gate, val), h, l);
    hi[r * ldo + c] = h;
    lo[r * ldo + c] = l;
  }
}

// ---------------------------------------------------------------------------------------------- trunk attention
struct TrunkAttnArgs {
  const float* q;
  int64_t ldq, q_bs;         // query (b, i) at q + b * q_bs + i * ldq + head * DH (q_bs = ldq = 0: one shared row)
  const float* k;
  const float* v;
  int64_t ldkv, kv_bs;       // key (b, j) at k + b * kv_bs + j * ldkv + head * DH
  const int32_t* q_grp;      // (B, Lq) option id of each query (OD_TRUNK_SELF)
  const int32_t* k_grp;      // (B, Lk) option id (SELF, CLS) or 0 (KEYS) per key; < 0 = padding
  const float* bonus;        // (H,) same-option bias (SELF)
  const int32_t* q_len;      // (B,) real queries / keys of each batch row (a prefix; the rest is padding), or null
  const int32_t* k_len;
  int mode, Lq, Lk, H, nqb;
  float scale;
  float* o;                  // (B * Lq, ldo) or null
  float* o_hi;               // the output's 3xTF32 operand pair, or null
  float* o_lo;
  int64_t ldo;
};

constexpr int TQ = 64;       // queries per CTA
constexpr int TKB = 64;      // keys per staged tile
constexpr int kAttnThreads = 256;   // 16 x 16: thread (ty, tx) holds rows ty + 16 i and keys tx + 16 j, i, j < 4

template <int DH>
struct AttnSmem {
  static constexpr int LD = DH + 4;                 // padded rows: 16 rows 16 apart fall on 8 distinct bank groups
  static constexpr int LP = TKB + 4;
  static constexpr int Q = 0, K = TQ * LD, V = K + 2 * TKB * LD, P = V + 2 * TKB * LD;
  static constexpr int floats = P + TQ * LP;
  static constexpr int bytes = floats * 4;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// A SIMT flash attention in fp32 with register tiles (q and k arrive RoPE'd: od_gemm_f32's epilogue rotates them).
// Per CTA: TQ queries of one (batch row, head); K / V tiles of TKB keys stream through shared memory by cp.async one
// tile ahead. S = Q K^T and O += P V are 4 x 4 register tiles per thread (8 FMAs per 16-byte shared load); the
// row max and the rescale of the online softmax are exchanged between the 16 threads of a row by shuffles. Keys past
// the row's real length are neither loaded nor counted; masked keys get probability 0.
template <int DH>
__global__ void __launch_bounds__(kAttnThreads, 2) trunk_attn_kernel(const TrunkAttnArgs a) {
  using L = AttnSmem<DH>;
  constexpr int LD = L::LD, LP = L::LP, CH = DH / 4, DPT = DH / 16;
  extern __shared__ __align__(16) float smem_f[];
  const int b = blockIdx.x / a.nqb, qb = blockIdx.x - b * a.nqb, h = blockIdx.y;
  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int lq = a.q_len ? min(max(a.q_len[b], 0), a.Lq) : a.Lq;   // padding queries past lq get zeros
  const int lk = a.k_len ? min(max(a.k_len[b], 0), a.Lk) : a.Lk;   // padding keys past lk are not read
  const int q0 = qb * TQ;
  auto out_row = [&](int i) { return (static_cast<int64_t>(b) * a.Lq + q0 + ty + 16 * i) * a.ldo + h * DH; };
  auto write = [&](int i, int d, float y) {
    const int64_t o = out_row(i) + d;
    if (a.o) a.o[o] = y;
    if (a.o_hi) {
      float hh, ll;
      split_tf32(y, hh, ll);
      a.o_hi[o] = hh;
      a.o_lo[o] = ll;
    }
  };
  if (q0 >= lq) {               // a block of padding queries (uniform over the CTA)
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (q0 + ty + 16 * i < a.Lq)
#pragma unroll
        for (int e = 0; e < DPT; ++e) write(i, tx * DPT + e, 0.f);
    return;
  }
  const uint32_t sbase = smem_u32(smem_f);
  const float* kb0 = a.k + b * a.kv_bs + h * DH;
  const float* vb0 = a.v + b * a.kv_bs + h * DH;
  auto stage = [&](int k0, int buf) {                 // keys k0 .. k0 + TKB - 1 into buffer buf
    const uint32_t ks = sbase + (L::K + buf * TKB * LD) * 4, vs = sbase + (L::V + buf * TKB * LD) * 4;
    for (int idx = t; idx < TKB * CH; idx += kAttnThreads) {
      const int j = idx / CH, c = (idx % CH) * 4;
      const bool ok = k0 + j < lk;
      const int64_t off = static_cast<int64_t>(ok ? k0 + j : 0) * a.ldkv + c;
      cp_async16(ks + (j * LD + c) * 4, kb0 + off, ok);
      cp_async16(vs + (j * LD + c) * 4, vb0 + off, ok);
    }
    cp_async_commit();
  };
  {   // the query block (rows past lq: zeros)
    const float* qb0 = a.q + b * a.q_bs + h * DH;
    for (int idx = t; idx < TQ * CH; idx += kAttnThreads) {
      const int r = idx / CH, c = (idx % CH) * 4;
      const bool ok = q0 + r < lq;
      cp_async16(sbase + (L::Q + r * LD + c) * 4, qb0 + static_cast<int64_t>(ok ? q0 + r : 0) * a.ldq + c, ok);
    }
  }
  if (lk > 0) stage(0, 0);    // commits the query block with the first tile
  else cp_async_commit();

  int qg[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qi = q0 + ty + 16 * i;
    qg[i] = a.mode == OD_TRUNK_SELF ? (qi < lq ? a.q_grp[static_cast<int64_t>(b) * a.Lq + qi] : -1) : qi;
  }
  const float bonus = a.mode == OD_TRUNK_SELF ? __ldg(a.bonus + h) : 0.f;
  const int32_t* kgrp = a.k_grp + static_cast<int64_t>(b) * a.Lk;

  float m[4], l[4], o[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < DPT; ++e) o[i][e] = 0.f;
  }
  const float* Qs = smem_f + L::Q;
  float* Ps = smem_f + L::P;

  for (int k0 = 0, buf = 0; k0 < lk; k0 += TKB, buf ^= 1) {
    if (k0 + TKB < lk) {
      stage(k0 + TKB, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* Ks = smem_f + L::K + buf * TKB * LD;
    const float* Vs = smem_f + L::V + buf * TKB * LD;

    // S = Q K^T: rows ty + 16 i, keys tx + 16 j, each an FMA chain over the head dimension in order
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int c = 0; c < DH; c += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * LD + c);
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * j) * LD + c);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
        }
    }
    // scale, bias and mask; the row max over the 16 threads of the row
    int gk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) gk[j] = k0 + tx + 16 * j < lk ? __ldg(kgrp + k0 + tx + 16 * j) : INT_MIN;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float rmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const bool ok = a.mode == OD_TRUNK_CLS ? gk[j] == qg[i] : gk[j] >= 0;
        float sc = __fmul_rn(s[i][j], a.scale);
        if (a.mode == OD_TRUNK_SELF && qg[i] >= 0 && gk[j] == qg[i]) sc = __fadd_rn(sc, bonus);
        s[i][j] = ok ? sc : -INFINITY;
        rmax = fmaxf(rmax, s[i][j]);
      }
#pragma unroll
      for (int x = 1; x < 16; x <<= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, x));
      const float mn = fmaxf(m[i], rmax);
      if (mn > m[i]) {                               // the same decision on the row's 16 threads
        const float f = expf(m[i] - mn);             // 0 while m is -inf
        l[i] *= f;
#pragma unroll
        for (int e = 0; e < DPT; ++e) o[i][e] *= f;
        m[i] = mn;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = s[i][j] == -INFINITY ? 0.f : expf(s[i][j] - m[i]);
        l[i] += p;
        Ps[(ty + 16 * i) * LP + tx + 16 * j] = p;
      }
    }
    __syncthreads();
    // O += P V: rows ty + 16 i, dims tx * DPT .. + DPT
#pragma unroll 4
    for (int kk = 0; kk < TKB; kk += 4) {
      float4 pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4*>(Ps + (ty + 16 * i) * LP + kk);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float vv[DPT];
        const float* vr = Vs + (kk + u) * LD + tx * DPT;
        if constexpr (DPT == 4) {
          const float4 x = *reinterpret_cast<const float4*>(vr);
          vv[0] = x.x;
          vv[1] = x.y;
          vv[2] = x.z;
          vv[3] = x.w;
        } else if constexpr (DPT == 2) {
          const float2 x = *reinterpret_cast<const float2*>(vr);
          vv[0] = x.x;
          vv[1] = x.y;
        } else {
          vv[0] = vr[0];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float p = u == 0 ? pv[i].x : u == 1 ? pv[i].y : u == 2 ? pv[i].z : pv[i].w;
#pragma unroll
          for (int e = 0; e < DPT; ++e) o[i][e] = fmaf(p, vv[e], o[i][e]);
        }
      }
    }
    __syncthreads();                                  // K / V / P buffers are rewritten next
  }
  cp_async_wait<0>();                                 // (no copy is left in flight when lk == 0)
  // the row sums over the 16 threads of the row, then O / l (a row with no visible key - a padded CLS option -
  // and a padding query get zeros)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int x = 1; x < 16; x <<= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], x);
    const int qi = q0 + ty + 16 * i;
    if (qi >= a.Lq) continue;
#pragma unroll
    for (int e = 0; e < DPT; ++e) write(i, tx * DPT + e, qi < lq && l[i] > 0.f ? __fdiv_rn(o[i][e], l[i]) : 0.f);
  }
}

// ---------------------------------------------------------------------------------------------- host helpers
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// (rows, cols) fp32 with row stride ld (elements) tiled into 32-column x 128-row boxes with the 128-byte swizzle;
// boxes past the tensor's edge are zero-filled
int make_map_f32(CUtensorMap* map, const float* base, uint64_t cols, uint64_t rows, uint64_t ld) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(FK), static_cast<cuuint32_t>(FB)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled (fp32 GEMM) failed (%d)", static_cast<int>(r));
  return OD_OK;
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!n[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev] = v > 0 ? v : 148;
  }
  return n[dev];
}

unsigned ew_blocks(int64_t n) {   // elementwise grids: enough 256-thread CTAs for ~8 waves, at least one
  const int64_t want = (n + 255) / 256, cap = 8LL * 16 * sm_count();
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

template <typename T>
int launch_scalenorm(const T* x, int64_t ldx, int64_t M, int K, const float* mixw, int n_mix, const float* g,
                     float eps, float* hi, float* lo, int64_t ldo, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(M));
#define OD_SN(V) scalenorm_split_kernel<T, V><<<grid, kNormThreads, 0, st>>>(x, ldx, K, mixw, n_mix, g, eps, hi, lo, ldo)
  if (K <= 128) OD_SN(1);
  else if (K <= 256) OD_SN(2);
  else if (K <= 512) OD_SN(4);
  else if (K <= 1024) OD_SN(8);
  else if (K <= 2048) OD_SN(16);
  else if (K <= 4096) OD_SN(32);
  else if (K <= 8192) OD_SN(64);
  else return fail(OD_EUNSUPPORTED, "od_scalenorm_split: K=%d above 8192", K);
#undef OD_SN
  OD_LAUNCH_CHECK();
  return ok();
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_split_tf32(const float* x, int64_t ldx, int64_t M, int64_t K, float* hi, float* lo, int64_t ldo,
                             void* stream) {
  OD_REQUIRE(x && hi && lo, "od_split_tf32: null pointer");
  OD_REQUIRE(M >= 0 && K > 0 && ldx >= K && ldo >= K, "od_split_tf32: bad shape");
  if (M == 0) return ok();
  split_tf32_kernel<<<ew_blocks(M * K), 256, 0, as_stream(stream)>>>(x, ldx, M, K, hi, lo, ldo);
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_scalenorm_split(const void* x, int dtype, int64_t ldx, int64_t M, int64_t K, const float* mix_w,
                                  int n_mix, const float* g, float eps, float* hi, float* lo, int64_t ldo,
                                  void* stream) {
  OD_REQUIRE(x && g && hi && lo, "od_scalenorm_split: null pointer");
  OD_REQUIRE(M >= 0 && M < (1LL << 31) && K > 0 && ldo >= K, "od_scalenorm_split: bad shape");
  OD_REQUIRE(mix_w ? (n_mix >= 1 && ldx >= n_mix * K) : ldx >= K, "od_scalenorm_split: row stride %lld too small",
             (long long)ldx);
  if (M == 0) return ok();
  cudaStream_t st = as_stream(stream);
  const int k = static_cast<int>(K);
  switch (dtype) {
    case OD_BF16:
      return launch_scalenorm(static_cast<const __nv_bfloat16*>(x), ldx, M, k, mix_w, n_mix, g, eps, hi, lo, ldo, st);
    case OD_F16:
      return launch_scalenorm(static_cast<const __half*>(x), ldx, M, k, mix_w, n_mix, g, eps, hi, lo, ldo, st);
    case OD_F32:
      return launch_scalenorm(static_cast<const float*>(x), ldx, M, k, mix_w, n_mix, g, eps, hi, lo, ldo, st);
    default:
      return fail(OD_EINVAL, "od_scalenorm_split: bad dtype %d", dtype);
  }
}

extern "C" int od_xatglu_split(const float* zv, int64_t ldzv, int64_t M, int64_t F, const float* alpha, float* hi,
                               float* lo, int64_t ldo, void* stream) {
  OD_REQUIRE(zv && alpha && hi && lo, "od_xatglu_split: null pointer");
  OD_REQUIRE(M >= 0 && F > 0 && ldzv >= 2 * F && ldo >= F, "od_xatglu_split: bad shape");
  if (M == 0) return ok();
  xatglu_split_kernel<<<ew_blocks(M * F), 256, 0, as_stream(stream)>>>(zv, ldzv, M, F, alpha, hi, lo, ldo);
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_gemm_f32(const float* x_hi, const float* x_lo, int64_t ldx, const float* w_hi, const float* w_lo,
                           int64_t ldw, const float* bias, const float* res, int64_t ldres, const int64_t* out_rows,
                           const int32_t* rope_pos, const float* rope_inv, int rope_cols, int rope_dh, float* y,
                           int64_t ldy, int64_t M, int64_t N, int64_t K, void* stream) {
  OD_REQUIRE(x_hi && x_lo && w_hi && w_lo && y, "od_gemm_f32: null pointer");
  OD_REQUIRE(M >= 0 && M < (1LL << 31) && N > 0 && N < (1LL << 31) && K > 0 && K % 4 == 0 && K < (1LL << 31),
             "od_gemm_f32: need K %% 4 == 0 (M=%lld N=%lld K=%lld)", (long long)M, (long long)N, (long long)K);
  OD_REQUIRE(ldx >= K && ldx % 4 == 0 && ldw >= K && ldw % 4 == 0 && ldy >= N && ldres >= 0,
             "od_gemm_f32: bad row strides (ldx %lld, ldw %lld, ldy %lld)", (long long)ldx, (long long)ldw,
             (long long)ldy);
  OD_REQUIRE(aligned16(x_hi) && aligned16(x_lo) && aligned16(w_hi) && aligned16(w_lo),
             "od_gemm_f32: operands must be 16-byte aligned");
  OD_REQUIRE(!rope_pos || (rope_inv && rope_dh >= 4 && rope_dh <= 128 && rope_dh % 4 == 0 && rope_cols >= 0 &&
                            rope_cols % rope_dh == 0 && rope_cols <= N),
             "od_gemm_f32: RoPE needs an even head width in [4, 128] (multiple of 4) dividing rope_cols <= N");
  if (M == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_gemm_f32: no device error word");
  CUtensorMap txh, txl, twh, twl;
  int rc = make_map_f32(&txh, x_hi, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(ldx));
  if (!rc) rc = make_map_f32(&txl, x_lo, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(ldx));
  if (!rc) rc = make_map_f32(&twh, w_hi, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldw));
  if (!rc) rc = make_map_f32(&twl, w_lo, static_cast<uint64_t>(K), static_cast<uint64_t>(N), static_cast<uint64_t>(ldw));
  if (rc) return rc;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(gemm_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem));
    attr[dev] = true;
  }
  GemmF32Args a;
  a.y = y;
  a.ldy = ldy;
  a.bias = bias;
  a.res = res;
  a.ldres = ldres;
  a.out_rows = out_rows;
  a.rope_pos = rope_pos;
  a.rope_inv = rope_inv;
  a.rope_cols = rope_pos ? rope_cols : 0;
  a.rope_dh = rope_pos ? rope_dh : 2;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.vec = ldy % 4 == 0 && aligned16(y) && (!res || (ldres % 4 == 0 && aligned16(res)));
  const int64_t tiles = ((M + FB - 1) / FB) * ((N + FB - 1) / FB);
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  gemm_f32_kernel<<<grid, kFThreads, kFSmem, as_stream(stream)>>>(txh, txl, twh, twl, a, err);
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_trunk_attn(const float* q, int64_t ldq, int64_t q_bstride, const float* k, const float* v,
                             int64_t ldkv, int64_t kv_bstride, const int32_t* q_grp, const int32_t* k_grp,
                             const float* bonus, const int32_t* q_len, const int32_t* k_len, int mode, int64_t B,
                             int64_t Lq, int64_t Lk, int H, int Dh, float* o, float* o_hi, float* o_lo, int64_t ldo,
                             void* stream) {
  OD_REQUIRE(q && k && v && k_grp && (o || (o_hi && o_lo)), "od_trunk_attn: null pointer");
  OD_REQUIRE(mode == OD_TRUNK_SELF || mode == OD_TRUNK_KEYS || mode == OD_TRUNK_CLS, "od_trunk_attn: bad mode %d",
             mode);
  OD_REQUIRE(mode != OD_TRUNK_SELF || (q_grp && bonus), "od_trunk_attn: self-attention needs q_grp and bonus");
  OD_REQUIRE(B >= 0 && Lq >= 0 && Lk >= 0 && H > 0 && Lq < (1LL << 30) && Lk < (1LL << 30),
             "od_trunk_attn: bad sizes");
  OD_REQUIRE(Dh == 16 || Dh == 32 || Dh == 64, "od_trunk_attn: head dim %d not in {16, 32, 64}", Dh);
  OD_REQUIRE(ldq % 4 == 0 && q_bstride % 4 == 0 && ldkv % 4 == 0 && kv_bstride % 4 == 0 && ldo >= H * Dh &&
                 aligned16(q) && aligned16(k) && aligned16(v),
             "od_trunk_attn: q / k / v rows must be 16-byte aligned");
  if (B == 0 || Lq == 0) return ok();
  TrunkAttnArgs a;
  a.q = q;
  a.ldq = ldq;
  a.q_bs = q_bstride;
  a.k = k;
  a.v = v;
  a.ldkv = ldkv;
  a.kv_bs = kv_bstride;
  a.q_grp = q_grp;
  a.k_grp = k_grp;
  a.bonus = bonus;
  a.q_len = q_len;
  a.k_len = k_len;
  a.mode = mode;
  a.Lq = static_cast<int>(Lq);
  a.Lk = static_cast<int>(Lk);
  a.H = H;
  a.nqb = static_cast<int>((Lq + TQ - 1) / TQ);
  a.scale = 1.0f / sqrtf(static_cast<float>(Dh));
  a.o = o;
  a.o_hi = o_hi;
  a.o_lo = o_lo;
  a.ldo = ldo;
  OD_REQUIRE(B * a.nqb < (1LL << 31) && H < 65536, "od_trunk_attn: grid too large");
  const dim3 grid(static_cast<unsigned>(B * a.nqb), static_cast<unsigned>(H));
  cudaStream_t st = as_stream(stream);
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(trunk_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     AttnSmem<64>::bytes));
    OD_CUDA_TRY(cudaFuncSetAttribute(trunk_attn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     AttnSmem<32>::bytes));
    OD_CUDA_TRY(cudaFuncSetAttribute(trunk_attn_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     AttnSmem<16>::bytes));
    attr[dev] = true;
  }
  switch (Dh) {
    case 16: trunk_attn_kernel<16><<<grid, kAttnThreads, AttnSmem<16>::bytes, st>>>(a); break;
    case 32: trunk_attn_kernel<32><<<grid, kAttnThreads, AttnSmem<32>::bytes, st>>>(a); break;
    default: trunk_attn_kernel<64><<<grid, kAttnThreads, AttnSmem<64>::bytes, st>>>(a); break;
  }
  OD_LAUNCH_CHECK();
  return ok();
}
