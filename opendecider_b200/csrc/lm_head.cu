// LM-head log-probability of given tokens: Backbone.token_logprob (backbone.py:165-178), the V3 trunk's option
// log-prob feature (v3_lm_feature, v3.py:437-442 and 527-532):
//     lp[m] = dot(float(h[m]), float(q[tok[m]]) * float(s[tok[m]])) - logsumexp_v float(bf16(h[m] . W[v]))
// with W = bf16(q * s) the tied head's rows as head_rows() dequantises them (quant.py:202-203). The vocabulary-wide
// normaliser never materialises M x V logits:
//   lm_lse_kernel   a bf16 tcgen05 GEMM of 128 rows of h against a contiguous range of the vocabulary (128 x 256
//                   tiles, K in 64-element blocks through a 4-stage TMA ring, two TMEM accumulators); its epilogue
//                   rounds each logit to bf16 (the reference's bf16 matmul output), keeps an online (max, sum of
//                   exp) per row across the CTA's tiles and writes one partial per row and vocabulary split
//   lm_merge_kernel one warp per row: the splits' partials merged by log-sum-exp, the target's fp32 dot product,
//                   their difference
// Vocabulary rows past V (the last tile's padding, zero-filled by TMA) are left out of the sums. Every wait is
// bounded: a time-out records an error code in the device error word and ends the kernel.
#include <cudaTypedefs.h>

#include "sm100.cuh"

namespace od {
namespace {
using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;   // BK bf16 = one 128-byte swizzle row
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kThreads = 192;                             // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int kSmemBytes = STAGES * STAGE_BYTES + 1024 /*barriers*/ + 1024 /*alignment slack*/;
constexpr int kMaxSplits = 32;                            // one partial per merge lane
constexpr int32_t kErrLm = 0x4C0000;

// 2^x (ex2.approx): the exponentials of the log-sum-exp in the base-2 domain
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// grid: vsplit x m_tiles CTAs, the split slowest, so the CTAs resident together read the same vocabulary tiles
// (each tile of W comes from HBM once per wave and from L2 for the other row tiles)
__global__ void __launch_bounds__(kThreads, 1)
    lm_lse_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int V,
                  int H, int tiles_per_split, int vsplit, float* __restrict__ part, int32_t* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM;
  const int split = blockIdx.x / m_tiles, mt = blockIdx.x % m_tiles;
  const int num_n = (V + BN - 1) / BN, num_kb = H / BK;
  const int t0 = split * tiles_per_split, t1 = min(num_n, t0 + tiles_per_split);
  const int m0 = mt * BM;

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
      uint32_t phase = 0, armed = 0, armed_par = 0;
      bool live = true;
      for (int nt = t0; nt < t1 && live; ++nt) {
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrLm | 1)) {
            live = false;
            break;
          }
          uint8_t* st_ = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(st_, &tmA, &full[stage], kb * BK, m0);
          tma_load_2d(st_ + A_BYTES, &tmB, &full[stage], kb * BK, nt * BN);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!live) {   // aborted: let the loads already issued land before shared memory goes away (bounded)
        for (int s = 0; s < STAGES; ++s)
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
      constexpr uint32_t idesc = idesc_bf16(BM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      bool live = true;
      for (int nt = t0, local = 0; nt < t1 && live; ++nt, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1, abort_flag, err, kErrLm | 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, err, kErrLm | 3)) {
            live = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16(d_tmem, desc_kmajor_sw128(a_addr + 32 * k), desc_kmajor_sw128(b_addr + 32 * k), idesc,
                    (kb | k) != 0);
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
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
    // ------------------------------------------------------------------ epilogue: online log-sum-exp per row
    const int quarter = warp & 3;                    // TMEM lanes 32 * quarter .. + 31 = tile rows
    const int row = m0 + quarter * 32 + lane;
    constexpr float kLog2e = 1.4426950408889634f;
    float run_max = -INFINITY, run_sum = 0.f;        // in log2 units: sum of 2^(x log2e - run_max)
    bool live = true;
    for (int nt = t0, local = 0; nt < t1; ++nt, ++local) {
      const int acc = local & 1;
      if (!mbar_wait(&tfull[acc], (local >> 1) & 1, abort_flag, err, kErrLm | 4)) {
        live = false;
        break;
      }
      tc_fence_after();
      const uint32_t tb = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int ncols = min(BN, V - nt * BN);        // real vocabulary columns of this tile
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tb + c * 32, r);
        tmem_ld_wait();
        float x[32];
        float cm = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          x[j] = c * 32 + j < ncols ? rbf(__uint_as_float(r[j])) * kLog2e : -INFINITY;
          cm = fmaxf(cm, x[j]);
        }
        if (cm > run_max) {
          run_sum = run_max == -INFINITY ? 0.f : run_sum * ex2f(run_max - cm);
          run_max = cm;
        }
        if (run_max != -INFINITY) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) s += ex2f(x[j] - run_max);
          run_sum += s;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (live && row < M) {
      float* dst = part + (static_cast<int64_t>(row) * vsplit + split) * 2;
      dst[0] = run_max;                               // log2 units
      dst[1] = run_sum;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// One warp per row: lse (natural log) from the splits' partials, the target logit in fp32, lp = target - lse.
__global__ void __launch_bounds__(256) lm_merge_kernel(const float* __restrict__ part, int vsplit,
                                                       const __nv_bfloat16* __restrict__ h, int H,
                                                       const int8_t* __restrict__ qW, const __nv_bfloat16* __restrict__ sW,
                                                       const int64_t* __restrict__ tok, int64_t V, int M,
                                                       float* __restrict__ lp) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float pm = -INFINITY, ps = 0.f;
  if (lane < vsplit) {
    pm = part[(row * vsplit + lane) * 2];
    ps = part[(row * vsplit + lane) * 2 + 1];
  }
  float gm = pm;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, o));
  float w = pm == -INFINITY ? 0.f : ps * ex2f(pm - gm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
  const int64_t t = tok[row];
  float dot = 0.f;
  if (t >= 0 && t < V) {
    const float s = __bfloat162float(sW[t]);
    const __nv_bfloat16* hr = h + row * H;
    const int8_t* qr = qW + t * H;
    for (int k = lane; k < H; k += 32)
      dot = fmaf(__bfloat162float(hr[k]), __fmul_rn(static_cast<float>(qr[k]), s), dot);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) {
    const float lse = (gm + log2f(w)) * 0.6931471805599453f;
    lp[row] = (t >= 0 && t < V && gm != -INFINITY) ? dot - lse : -INFINITY;
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

// (rows, cols) bf16 row-major tiled into BK-column x box_rows boxes with the 128-byte swizzle
int make_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled (lm head) failed (%d)", static_cast<int>(r));
  return OD_OK;
}

// vocabulary splits: enough CTAs for about 6 waves, at most kMaxSplits
int plan_vsplit(int64_t M, int64_t V, int num_sms) {
  const int64_t m_tiles = (M + BM - 1) / BM, n_tiles = (V + BN - 1) / BN;
  int64_t s = (6LL * (num_sms > 0 ? num_sms : 148) + m_tiles - 1) / m_tiles;
  if (s > kMaxSplits) s = kMaxSplits;
  if (s > n_tiles) s = n_tiles;
  return static_cast<int>(s < 1 ? 1 : s);
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_lm_logprob_plan(int64_t M, int64_t V, int num_sms, int* vsplit, int64_t* workspace_bytes) {
  OD_REQUIRE(vsplit && workspace_bytes, "od_lm_logprob_plan: null pointer");
  OD_REQUIRE(M >= 0 && V > 0, "od_lm_logprob_plan: bad sizes");
  *vsplit = plan_vsplit(M, V, num_sms);
  *workspace_bytes = static_cast<int64_t>(sizeof(float)) * 2 * M * *vsplit;
  return ok();
}

extern "C" int od_lm_logprob(const void* h, int64_t M, int H, const void* Wb, const int8_t* qW, const void* sW,
                             int64_t V, const int64_t* tok, float* lp, void* workspace, int64_t workspace_bytes,
                             int vsplit, void* stream) {
  OD_REQUIRE(h && Wb && qW && sW && tok && lp && workspace, "od_lm_logprob: null pointer");
  OD_REQUIRE(M >= 0 && M < (1LL << 31) && V > 0 && V < (1LL << 31), "od_lm_logprob: bad sizes");
  OD_REQUIRE(H > 0 && H % BK == 0, "od_lm_logprob: hidden %d must be a multiple of %d", H, BK);
  OD_REQUIRE(vsplit >= 1 && vsplit <= kMaxSplits, "od_lm_logprob: vsplit %d not in [1, %d]", vsplit, kMaxSplits);
  OD_REQUIRE(workspace_bytes >= static_cast<int64_t>(sizeof(float)) * 2 * M * vsplit,
             "od_lm_logprob: workspace below 8 x M x vsplit bytes (od_lm_logprob_plan)");
  OD_REQUIRE(aligned16(h) && aligned16(Wb) && aligned16(workspace), "od_lm_logprob: tensors must be 16-byte aligned");
  if (M == 0) return ok();
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_lm_logprob: no device error word");
  CUtensorMap ta, tb;
  int rc = make_map(&ta, h, static_cast<uint64_t>(H), static_cast<uint64_t>(M), BM);
  if (!rc) rc = make_map(&tb, Wb, static_cast<uint64_t>(H), static_cast<uint64_t>(V), BN);
  if (rc) return rc;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(lm_lse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    attr[dev] = true;
  }
  cudaStream_t st = as_stream(stream);
  const int m_tiles = static_cast<int>((M + BM - 1) / BM);
  const int n_tiles = static_cast<int>((V + BN - 1) / BN);
  const int tps = (n_tiles + vsplit - 1) / vsplit;
  OD_REQUIRE(static_cast<int64_t>(m_tiles) * vsplit < (1LL << 31), "od_lm_logprob: grid too large");
  float* part = static_cast<float*>(workspace);
  lm_lse_kernel<<<m_tiles * vsplit, kThreads, kSmemBytes, st>>>(ta, tb, static_cast<int>(M), static_cast<int>(V), H,
                                                                  tps, vsplit, part, err);
  OD_LAUNCH_CHECK();
  const unsigned mb = static_cast<unsigned>((M * 32 + 255) / 256);
  lm_merge_kernel<<<mb, 256, 0, st>>>(part, vsplit, static_cast<const __nv_bfloat16*>(h), H, qW,
                                      static_cast<const __nv_bfloat16*>(sW), tok, V, static_cast<int>(M), lp);
  OD_LAUNCH_CHECK();
  return ok();
}
