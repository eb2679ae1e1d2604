// W8A8 GEMM on the sm_100a 5th-generation tensor cores (the int8 projections q/k/v/o, gate/up, down).
//
//   acc[m, n] = sum_k A[m, k] * W[n, k]     int8 x int8 -> int32, exact, accumulated in TMEM
//   Y[m, n]   = bf16((float(acc) * sa[m]) * float(sw[n]))   or the fused SwiGLU / raw int32 epilogues
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised):
//   warp 0    TMA producer: 128x128 A tile + 256x128 W tile per k-block into a 4-stage ring (48 KB/stage),
//             128-byte swizzle, no multicast (every CTA issues its own loads).
//   warp 1    MMA issuer: four tcgen05.mma.kind::i8 (M=128, N=256, K=32) per k-block into one of two TMEM
//             accumulators (2 x 256 columns = all 512 columns), tcgen05.commit frees the smem stage.
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (each warp its 32-lane TMEM quarter = 32 rows), scale,
//             round, store; the second accumulator lets the next tile's MMAs overlap this epilogue.
// Tiles run n-fastest, so the CTAs working at the same time share A rows and the whole weight stays in L2.
#include <cudaTypedefs.h>

#include "sm100.cuh"

namespace od {
namespace {
using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + 1024 /*barriers*/ + 1024 /*alignment slack*/;

// error codes written to the device error word (high half identifies the kernel, low half the wait)
constexpr int32_t kErrGemm = 0x6E0000;

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
    reinterpret_cast<uint4*>(dst)[i] = raw;
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(src) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[8 * i + 2 * j] = f.x;
      v[8 * i + 2 * j + 1] = f.y;
    }
  }
}

// Epilogue of one 128 x 256 accumulator in TMEM (tbase: this warp's lane quarter): this thread's output row m,
// columns n0 .. n0 + 255 (SwiGLU: outputs tile_n * 128 .. + 127); rows of Y are ldy elements apart. Columns at or
// beyond N (a last tile wider than the weight: its rows were zero-filled by TMA) are not stored.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, int m, bool valid, int n0, int tile_n,
                                              const float* __restrict__ sa, const __nv_bfloat16* __restrict__ sw,
                                              void* __restrict__ Y, int64_t ldy, int N) {
  const float sam = valid ? sa[m] : 0.f;
  if constexpr (EPI == OD_EPI_INT32) {
#pragma unroll 1
    for (int c = 0; c < BN / 32 && n0 + c * 32 < N; ++c) {        // warp-uniform bound (tcgen05.ld is collective)
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c * 32, r);
      tmem_ld_wait();
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<int32_t*>(Y) + static_cast<int64_t>(m) * ldy + n0 + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      }
    }
  } else if constexpr (EPI == OD_EPI_BF16) {
#pragma unroll 1
    for (int c = 0; c < BN / 32 && n0 + c * 32 < N; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c * 32, r);
      tmem_ld_wait();
      if (valid) {
        float w[32], y[32];
        load_bf16x32(sw + n0 + c * 32, w);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          y[j] = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(r[j])), sam), w[j]);
        store_bf16x32(static_cast<__nv_bfloat16*>(Y) + static_cast<int64_t>(m) * ldy + n0 + c * 32, y);
      }
    }
  } else {  // OD_EPI_SWIGLU: columns [0,128) gate, [128,256) up of the same 128 outputs
    const int j0 = tile_n * (BN / 2);
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t rg[32], ru[32];
      tmem_ld_32x32b_x32(tbase + c * 32, rg);
      tmem_ld_32x32b_x32(tbase + BN / 2 + c * 32, ru);
      tmem_ld_wait();
      if (valid) {
        float wg[32], wu[32], y[32];
        load_bf16x32(sw + n0 + c * 32, wg);
        load_bf16x32(sw + n0 + BN / 2 + c * 32, wu);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float g = rbf(__fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(rg[j])), sam), wg[j]));
          const float u = rbf(__fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(ru[j])), sam), wu[j]));
          const float a = rbf(__fdiv_rn(g, 1.0f + expf(-g)));  // SiLU in fp32, stored as bf16
          y[j] = __fmul_rn(a, u);
        }
        store_bf16x32(static_cast<__nv_bfloat16*>(Y) + static_cast<int64_t>(m) * ldy + j0 + c * 32, y);
      }
    }
  }
}

// Split-K (single-CTA form, small M): the K range of a tile is divided among `splits` work items, each of which
// writes its int32 partial tile to the workspace (tiles x splits x BM x BN); a second kernel sums the partials -
// exact, integer addition - and runs the epilogue, one thread per 8 outputs. No CTA waits for another.
struct SplitK {
  int splits;
  int32_t* part;
};

template <int EPI>
__global__ void __launch_bounds__(256) gemm_splitk_reduce_kernel(const int32_t* __restrict__ part, int splits, int M,
                                                                 int N, const float* __restrict__ sa,
                                                                 const __nv_bfloat16* __restrict__ sw,
                                                                 void* __restrict__ Y, int64_t ldy) {
  const int num_n = (N + BN - 1) / BN;
  const int groups = EPI == OD_EPI_SWIGLU ? N / 16 : N / 8;     // 8-output groups per row
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(M) * groups) return;
  const int m = static_cast<int>(idx / groups), gi = static_cast<int>(idx % groups);
  const int row = m % BM;
  // accumulator columns of this group: BF16 / INT32 output n = 8 gi .. + 7; SwiGLU outputs j = 8 gi .. + 7 read the
  // gate columns c and the up columns BN / 2 + c of their tile
  const int n = EPI == OD_EPI_SWIGLU ? (gi * 8 / (BN / 2)) * BN + (gi * 8) % (BN / 2) : gi * 8;
  const int tile = (m / BM) * num_n + n / BN, col = n % BN;
  int32_t a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, u[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int sp = 0; sp < splits; ++sp) {
    const int32_t* src = part + ((static_cast<int64_t>(tile) * splits + sp) * BM + row) * BN + col;
    const int4 x0 = __ldcg(reinterpret_cast<const int4*>(src)), x1 = __ldcg(reinterpret_cast<const int4*>(src) + 1);
    a[0] += x0.x; a[1] += x0.y; a[2] += x0.z; a[3] += x0.w; a[4] += x1.x; a[5] += x1.y; a[6] += x1.z; a[7] += x1.w;
    if constexpr (EPI == OD_EPI_SWIGLU) {
      const int4 y0 = __ldcg(reinterpret_cast<const int4*>(src + BN / 2));
      const int4 y1 = __ldcg(reinterpret_cast<const int4*>(src + BN / 2) + 1);
      u[0] += y0.x; u[1] += y0.y; u[2] += y0.z; u[3] += y0.w; u[4] += y1.x; u[5] += y1.y; u[6] += y1.z; u[7] += y1.w;
    }
  }
  if constexpr (EPI == OD_EPI_INT32) {
    int4* dst = reinterpret_cast<int4*>(static_cast<int32_t*>(Y) + static_cast<int64_t>(m) * ldy + n);
    dst[0] = make_int4(a[0], a[1], a[2], a[3]);
    dst[1] = make_int4(a[4], a[5], a[6], a[7]);
  } else {
    const float sam = sa[m];
    float y[8];
    if constexpr (EPI == OD_EPI_BF16) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        y[j] = __fmul_rn(__fmul_rn(static_cast<float>(a[j]), sam), __bfloat162float(sw[n + j]));
    } else {                                           // the OD_EPI_SWIGLU epilogue's rounding points
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = rbf(__fmul_rn(__fmul_rn(static_cast<float>(a[j]), sam), __bfloat162float(sw[n + j])));
        const float v = rbf(__fmul_rn(__fmul_rn(static_cast<float>(u[j]), sam), __bfloat162float(sw[n + BN / 2 + j])));
        y[j] = __fmul_rn(rbf(__fdiv_rn(g, 1.0f + expf(-g))), v);
      }
    }
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
    const int64_t out_col = EPI == OD_EPI_SWIGLU ? static_cast<int64_t>(gi) * 8 : n;
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(Y) + static_cast<int64_t>(m) * ldy + out_col) = w;
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const float* __restrict__ sa, const __nv_bfloat16* __restrict__ sw, void* __restrict__ Y, int M,
                     int N, int K, int64_t ldy, int32_t* err, SplitK sk) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // pointer arithmetic on the shared array (not an integer cast) keeps the shared address space visible
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN, num_kb = K / BK;
  const int num_tiles = num_m * num_n;
  const int splits = sk.splits;
  const int num_items = num_tiles * splits;               // item = tile x splits + split

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0;  // bit s: stage s holds a load issued with parity bit (armed_par >> s) & 1
      uint32_t armed_par = 0;
      bool live = true;
      for (int item = blockIdx.x; item < num_items && live; item += gridDim.x) {
        const int tile = item / splits, sp = item - tile * splits;
        const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
        const int kb0 = sp * num_kb / splits, kb1 = (sp + 1) * num_kb / splits;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrGemm | 1)) {
            live = false;
            break;
          }
          uint8_t* sa_ = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(sa_, &tmA, &full[stage], kb * BK, m0);
          tma_load_2d(sa_ + A_BYTES, &tmB, &full[stage], kb * BK, n0);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!live) {
        // aborted: let the loads already issued land before the CTA's shared memory goes away (bounded)
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], (armed_par >> s) & 1) && clock64() - t0 < kWaitLimitCycles) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool live = true;
      for (int item = blockIdx.x; item < num_items && live; item += gridDim.x, ++local) {
        const int sp = item % splits;
        const int kb0 = sp * num_kb / splits, kb1 = (sp + 1) * num_kb / splits;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, err, kErrGemm | 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, err, kErrGemm | 3)) {
            live = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8(d_tmem, desc_kmajor_sw128(a_addr + 32 * k), desc_kmajor_sw128(b_addr + 32 * k), idesc,
                   (kb != kb0 || k != 0));
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (live) mma_commit(&tfull[acc]);
      }
      // every MMA this thread issued has completed before TMEM is released (immediate unless aborted)
      mma_commit(drain);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitLimitCycles) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32) = tile rows
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x, ++local) {
      const int tile = item / splits, sp = item - tile * splits;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, err, kErrGemm | 4)) break;
      tc_fence_after();
      const int m = (tile / num_n) * BM + row;
      const int n0 = (tile % num_n) * BN;
      const bool valid = m < M;
      const uint32_t tacc = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (splits == 1) {
        epilogue_tile<EPI>(tacc, m, valid, n0, tile % num_n, sa, sw, Y, ldy, N);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
      // split-K: this item's partial accumulator row into the workspace (summed by gemm_splitk_reduce_kernel)
      int32_t* mine = sk.part + ((static_cast<int64_t>(tile) * splits + sp) * BM + row) * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tacc + c * 32, r);
        tmem_ld_wait();
        uint4* dst = reinterpret_cast<uint4*>(mine + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) __stcg(dst + i, make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}


// ------------------------------------------------------------------------------------------------ CTA-pair form
// Large M: a cluster of two CTAs computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256). Each CTA stages
// 128 rows of A and 128 rows of W per k-block (32 KB per stage instead of 48 KB for a 128 x 256 tile: the shared-
// memory operand traffic per MAC, which bounds the single-CTA form, drops by a third) and holds 128 rows x 256
// columns of the accumulator in its own TMEM. Both CTAs' loads of a stage complete on the even CTA's stage barrier,
// which the even CTA arms for both CTAs' bytes (a remote arrival per stage from the odd CTA would serialise its
// loads); its single thread issues the pair's MMAs and multicasts its
// commits (stage free, accumulator full) to both CTAs; the epilogue warps of both CTAs release an accumulator on the
// even CTA's barrier. Barriers that complete through the other CTA are polled without a suspend hint. After a
// time-out the even CTA completes and waits for every stage phase either CTA armed, so no load is in flight when the
// pair leaves (the final cluster barrier holds the odd CTA until then).
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK, P_B_BYTES = 128 * BK, P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int kPairSmemBytes = P_STAGES * P_STAGE_BYTES + 1024 /*barriers*/ + 1024 /*alignment slack*/;
constexpr int PM = 256;   // rows per pair tile

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const float* __restrict__ sa, const __nv_bfloat16* __restrict__ sw, void* __restrict__ Y,
                          int M, int N, int K, int64_t ldy, int32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_m = (M + PM - 1) / PM, num_n = (N + BN - 1) / BN, num_kb = K / BK;
  const int num_tiles = num_m * num_n;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full[s], 1);                         // (even CTA) armed for both CTAs' bytes
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);                       // the 4 epilogue warps of both CTAs (used on the even CTA)
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, kTmemCols);
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync();                                     // both CTAs' barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_par = 0;
      bool live = true;
      for (int tile = pair; tile < num_tiles && live; tile += num_pairs) {
        const int m0 = (tile / num_n) * PM + static_cast<int>(rank) * 128;
        const int n0 = (tile % num_n) * BN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_spin(&empty[stage], phase ^ 1, abort_flag, err, kErrGemm | 0x11)) {
            live = false;
            break;
          }
          uint8_t* st_ = smem + stage * P_STAGE_BYTES;
          const uint32_t fb = mapa_shared(&full[stage], 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          tma_load_2d_pair(st_, &tmA, fb, kb * BK, m0);
          tma_load_2d_pair(st_ + P_A_BYTES, &tmB, fb, kb * BK, n0);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!live && leader) {
        // aborted: every stage's last armed phase, and the phase after it (for which the odd CTA may have issued its
        // loads alone: arming it for the odd CTA's bytes lets it complete once they land), must be complete before
        // the pair leaves
        constexpr long long kDrainCycles = 4000000;   // about 2 ms: an issued load lands well within it
        for (int s = 0; s < P_STAGES; ++s) {
          const uint32_t last = (armed >> s) & 1 ? (armed_par >> s) & 1 : 1;
          if ((armed >> s) & 1) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&full[s], last) && clock64() - t0 < kDrainCycles) {
            }
          }
          mbar_arrive_expect_tx(&full[s], P_STAGE_BYTES);
          const long long t0 = clock64();
          while (!mbar_try_wait(&full[s], last ^ 1) && clock64() - t0 < kDrainCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------------------------------------------- MMA issuer of the pair (even CTA)
      constexpr uint32_t idesc = idesc_i8(PM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool live = true;
      for (int tile = pair; tile < num_tiles && live; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_spin(&tempty[acc], acc_phase ^ 1, abort_flag, err, kErrGemm | 0x12)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_spin(&full[stage], phase, abort_flag, err, kErrGemm | 0x13)) {
            live = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint32_t b_addr = a_addr + P_A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8_pair(d_tmem, desc_kmajor_sw128(a_addr + 32 * k), desc_kmajor_sw128(b_addr + 32 * k), idesc,
                        (kb | k) != 0);
          mma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (live) mma_commit_pair(&tfull[acc], 0x3);
      }
      mma_commit_pair(drain, 0x1);
      const long long t0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - t0 < kWaitLimitCycles) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5 of both CTAs)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t tempty_even[2] = {mapa_shared(&tempty[0], 0), mapa_shared(&tempty[1], 0)};
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_spin(&tfull[acc], acc_phase, abort_flag, err, kErrGemm | 0x15)) break;
      tc_fence_after();
      const int m = (tile / num_n) * PM + static_cast<int>(rank) * 128 + row;
      epilogue_tile<EPI>(tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16), m, m < M,
                         (tile % num_n) * BN, tile % num_n, sa, sw, Y, ldy, N);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_even[acc]);
    }
  }

  __syncthreads();
  cluster_sync();                                     // the pair's MMAs are drained; no cross-CTA access remains
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------------ host side
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

// A 2-D int8 tensor (outer rows of `inner` bytes) tiled into box_outer x box_inner boxes, 128-byte swizzle.
int make_map_i8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_inner,
                uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return OD_OK;
}

int num_sms() {
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

template <int EPI>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const float* sa, const __nv_bfloat16* sw, void* Y,
                int M, int N, int K, int64_t ldy, int32_t* err, cudaStream_t st, SplitK sk = SplitK{1, nullptr}) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[dev] = true;
  }
  const int items = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * sk.splits;
  const int grid = items < num_sms() ? items : num_sms();
  gemm_w8a8_kernel<EPI><<<grid, kThreads, kSmemBytes, st>>>(ta, tb, sa, sw, Y, M, N, K, ldy, err, sk);
  OD_LAUNCH_CHECK();
  return ok();
}

template <int EPI>
int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const float* sa, const __nv_bfloat16* sw, void* Y,
                     int M, int N, int K, int64_t ldy, int32_t* err, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_pair_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kPairSmemBytes));
    attr_set[dev] = true;
  }
  const int tiles = ((M + PM - 1) / PM) * ((N + BN - 1) / BN);
  const int pairs = tiles < num_sms() / 2 ? tiles : num_sms() / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  OD_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_w8a8_pair_kernel<EPI>, ta, tb, sa, sw, Y, M, N, K, ldy, err));
  OD_LAUNCH_CHECK();
  return ok();
}

// rows from which the CTA-pair form is used (below it the single-CTA tiles give more CTAs to small problems)
constexpr int64_t kPairMinRows = 1024;

}  // namespace
}  // namespace od

using namespace od;

namespace od {
namespace {
// Split count of the single-CTA form for a small-M problem, in units of one k-block per wave of CTAs: (waves of work
// items) x (k-blocks per item + about 2 of fixed cost), plus, when split, the partial tiles' round trip through L2 and
// the reduction launch (measured on B200 at about 4 units + 0.17 per partial tile: 17 us for 128). Splitting pays
// only for long K (M = 512, K = 12288: 45.7 us against 51.8); at most 8 splits and at most the k-blocks.
int plan_splits_gemm(int64_t M, int64_t N, int64_t K, int sms) {
  if (M >= kPairMinRows || sms <= 0) return 1;
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int64_t kb = K / BK;
  int best = 1;
  double best_t = 1e300;
  for (int s = 1; s <= 8 && s <= kb; ++s) {
    const double waves = static_cast<double>((tiles * s + sms - 1) / sms);
    const double t = waves * (static_cast<double>((kb + s - 1) / s) + 2.0) + (s > 1 ? 4.0 + 0.17 * tiles * s : 0.0);
    if (t < best_t * 0.97) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

int64_t splitk_bytes(int64_t M, int64_t N, int splits) {
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  return tiles * splits * BM * BN * static_cast<int64_t>(sizeof(int32_t));
}

int gemm_entry(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y, int64_t M, int64_t N,
               int64_t K, int epilogue, int64_t ldy, int splits, void* workspace, int64_t workspace_bytes,
               void* stream) {
  OD_REQUIRE(A && W && Y, "od_gemm_w8a8: null pointer");
  OD_REQUIRE(epilogue == OD_EPI_INT32 || (sa && sw), "od_gemm_w8a8: scales are required for this epilogue");
  OD_REQUIRE(M >= 0 && M < (1LL << 31) && N > 0 && N % (epilogue == OD_EPI_SWIGLU ? BN : 32) == 0 &&
                 N < (1LL << 31) && K > 0 && K % BK == 0 && K < (1LL << 31),
             "od_gemm_w8a8: need N %% 32 == 0 (SwiGLU: N %% 256 == 0) and K %% 128 == 0 (M=%lld N=%lld K=%lld)",
             (long long)M, (long long)N, (long long)K);
  OD_REQUIRE(aligned16(A) && aligned16(W) && aligned16(Y), "od_gemm_w8a8: A, W, Y must be 16-byte aligned");
  OD_REQUIRE(epilogue >= OD_EPI_BF16 && epilogue <= OD_EPI_INT32, "od_gemm_w8a8: bad epilogue %d", epilogue);
  const int64_t cols = epilogue == OD_EPI_SWIGLU ? N / 2 : N;
  const int64_t vec = epilogue == OD_EPI_INT32 ? 4 : 8;          // elements of one 16-byte store
  OD_REQUIRE(ldy >= cols && ldy % vec == 0 && ldy < (1LL << 40),
             "od_gemm_w8a8: output row stride %lld must be >= %lld and a multiple of %lld elements", (long long)ldy,
             (long long)cols, (long long)vec);
  const bool pairs = M >= kPairMinRows;
  OD_REQUIRE(splits >= 1 && splits <= 8 && splits <= K / BK, "od_gemm_w8a8: splits %d must be in [1, min(8, K/128)]",
             splits);
  OD_REQUIRE(splits == 1 || !pairs, "od_gemm_w8a8: split-K is for M < %lld (the single-CTA form)",
             (long long)kPairMinRows);
  if (splits > 1)
    OD_REQUIRE(workspace && aligned16(workspace) && workspace_bytes >= splitk_bytes(M, N, splits),
               "od_gemm_w8a8: %d splits need a 16-byte aligned workspace of %lld bytes (od_gemm_w8a8_plan)",
               splits, (long long)splitk_bytes(M, N, splits));
  if (M == 0) return ok();
  CUtensorMap ta, tb;
  int rc = make_map_i8(&ta, A, static_cast<uint64_t>(K), static_cast<uint64_t>(M), BK, BM);
  if (rc) return rc;
  rc = make_map_i8(&tb, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N), BK, pairs ? 128 : BN);
  if (rc) return rc;
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_gemm_w8a8: no device error word");
  cudaStream_t st = as_stream(stream);
  const auto swp = static_cast<const __nv_bfloat16*>(sw);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  if (pairs) {
    switch (epilogue) {
      case OD_EPI_BF16: return launch_gemm_pair<OD_EPI_BF16>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st);
      case OD_EPI_SWIGLU: return launch_gemm_pair<OD_EPI_SWIGLU>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st);
      default: return launch_gemm_pair<OD_EPI_INT32>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st);
    }
  }
  SplitK sk{splits, static_cast<int32_t*>(workspace)};
  switch (epilogue) {
    case OD_EPI_BF16: rc = launch_gemm<OD_EPI_BF16>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st, sk); break;
    case OD_EPI_SWIGLU: rc = launch_gemm<OD_EPI_SWIGLU>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st, sk); break;
    default: rc = launch_gemm<OD_EPI_INT32>(ta, tb, sa, swp, Y, m, n, k, ldy, err, st, sk); break;
  }
  if (rc != OD_OK || splits == 1) return rc;
  const int64_t threads = M * (epilogue == OD_EPI_SWIGLU ? N / 16 : N / 8);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  const int32_t* part = static_cast<const int32_t*>(workspace);
  switch (epilogue) {
    case OD_EPI_BF16: gemm_splitk_reduce_kernel<OD_EPI_BF16><<<blocks, 256, 0, st>>>(part, splits, m, n, sa, swp, Y, ldy); break;
    case OD_EPI_SWIGLU: gemm_splitk_reduce_kernel<OD_EPI_SWIGLU><<<blocks, 256, 0, st>>>(part, splits, m, n, sa, swp, Y, ldy); break;
    default: gemm_splitk_reduce_kernel<OD_EPI_INT32><<<blocks, 256, 0, st>>>(part, splits, m, n, sa, swp, Y, ldy); break;
  }
  OD_LAUNCH_CHECK();
  return ok();
}
}  // namespace
}  // namespace od

extern "C" int od_gemm_w8a8_ld(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y, int64_t M,
                               int64_t N, int64_t K, int epilogue, int64_t ldy, void* stream) {
  return gemm_entry(A, sa, W, sw, Y, M, N, K, epilogue, ldy, 1, nullptr, 0, stream);
}

extern "C" int od_gemm_w8a8_plan(int64_t M, int64_t N, int64_t K, int num_sms, int* splits, int64_t* workspace_bytes) {
  OD_REQUIRE(splits && workspace_bytes && M >= 0 && N > 0 && K > 0, "od_gemm_w8a8_plan: bad arguments");
  *splits = plan_splits_gemm(M, N, K, num_sms);
  *workspace_bytes = *splits > 1 ? splitk_bytes(M, N, *splits) : 0;
  return ok();
}

extern "C" int od_gemm_w8a8_splitk(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y,
                                   int64_t M, int64_t N, int64_t K, int epilogue, int64_t ldy, int splits,
                                   void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_entry(A, sa, W, sw, Y, M, N, K, epilogue, ldy, splits, workspace, workspace_bytes, stream);
}

extern "C" int od_gemm_w8a8(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y, int64_t M,
                            int64_t N, int64_t K, int epilogue, void* stream) {
  return od_gemm_w8a8_ld(A, sa, W, sw, Y, M, N, K, epilogue, epilogue == OD_EPI_SWIGLU ? N / 2 : N, stream);
}
