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

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const float* __restrict__ sa, const __nv_bfloat16* __restrict__ sw, void* __restrict__ Y, int M,
                     int N, int K, int32_t* err) {
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
  const int num_m = (M + BM - 1) / BM, num_n = N / BN, num_kb = K / BK;
  const int num_tiles = num_m * num_n;

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
      for (int tile = blockIdx.x; tile < num_tiles && live; tile += gridDim.x) {
        const int m0 = (tile / num_n) * BM, n0 = (tile % num_n) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
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
      for (int tile = blockIdx.x; tile < num_tiles && live; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, err, kErrGemm | 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
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
                   (kb | k) != 0);
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
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, err, kErrGemm | 4)) break;
      tc_fence_after();
      const int m = (tile / num_n) * BM + row;
      const int n0 = (tile % num_n) * BN;
      const bool valid = m < M;
      const float sam = valid ? sa[m] : 0.f;
      const uint32_t tbase = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if constexpr (EPI == OD_EPI_INT32) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<int32_t*>(Y) + static_cast<int64_t>(m) * N + n0 + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
          }
        }
      } else if constexpr (EPI == OD_EPI_BF16) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_ld_wait();
          if (valid) {
            float w[32], y[32];
            load_bf16x32(sw + n0 + c * 32, w);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              y[j] = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(r[j])), sam), w[j]);
            store_bf16x32(static_cast<__nv_bfloat16*>(Y) + static_cast<int64_t>(m) * N + n0 + c * 32, y);
          }
        }
      } else {  // OD_EPI_SWIGLU: columns [0,128) gate, [128,256) up of the same 128 outputs
        const int ldy = N / 2;
        const int j0 = (tile % num_n) * (BN / 2);
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
                int M, int N, int K, int32_t* err, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(gemm_w8a8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr_set[dev] = true;
  }
  const int tiles = ((M + BM - 1) / BM) * (N / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  gemm_w8a8_kernel<EPI><<<grid, kThreads, kSmemBytes, st>>>(ta, tb, sa, sw, Y, M, N, K, err);
  OD_LAUNCH_CHECK();
  return ok();
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_gemm_w8a8(const int8_t* A, const float* sa, const int8_t* W, const void* sw, void* Y, int64_t M,
                            int64_t N, int64_t K, int epilogue, void* stream) {
  OD_REQUIRE(A && W && Y, "od_gemm_w8a8: null pointer");
  OD_REQUIRE(epilogue == OD_EPI_INT32 || (sa && sw), "od_gemm_w8a8: scales are required for this epilogue");
  OD_REQUIRE(M >= 0 && M < (1LL << 31) && N > 0 && N % BN == 0 && N < (1LL << 31) && K > 0 && K % BK == 0 &&
                 K < (1LL << 31),
             "od_gemm_w8a8: need N %% 256 == 0 and K %% 128 == 0 (M=%lld N=%lld K=%lld)", (long long)M, (long long)N,
             (long long)K);
  OD_REQUIRE(aligned16(A) && aligned16(W) && aligned16(Y), "od_gemm_w8a8: A, W, Y must be 16-byte aligned");
  OD_REQUIRE(epilogue >= OD_EPI_BF16 && epilogue <= OD_EPI_INT32, "od_gemm_w8a8: bad epilogue %d", epilogue);
  if (M == 0) return ok();
  CUtensorMap ta, tb;
  int rc = make_map_i8(&ta, A, static_cast<uint64_t>(K), static_cast<uint64_t>(M), BK, BM);
  if (rc) return rc;
  rc = make_map_i8(&tb, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N), BK, BN);
  if (rc) return rc;
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_gemm_w8a8: no device error word");
  cudaStream_t st = as_stream(stream);
  const auto swp = static_cast<const __nv_bfloat16*>(sw);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  switch (epilogue) {
    case OD_EPI_BF16: return launch_gemm<OD_EPI_BF16>(ta, tb, sa, swp, Y, m, n, k, err, st);
    case OD_EPI_SWIGLU: return launch_gemm<OD_EPI_SWIGLU>(ta, tb, sa, swp, Y, m, n, k, err, st);
    default: return launch_gemm<OD_EPI_INT32>(ta, tb, sa, swp, Y, m, n, k, err, st);
  }
}
