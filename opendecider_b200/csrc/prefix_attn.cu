// Branched shared-prefix attention on the sm_100a tensor cores (the Hydragen split of prefix_attn._split_attention,
// merged exactly by log-sum-exp, here as one online softmax over the three key segments of a query row).
//
// One CTA = 128 query slots (one per TMEM lane) of one KV head: the slots are (row, token, head of the GQA group) of
// a row group - one long row (the state pass: 32 tokens x 4 heads per CTA) or several short rows of the same question
// (option rows), so the tensor-core tile is filled and each prefix block staged once serves all of them. Keys run in
// blocks of 128 through a warp-specialised pipeline:
//   producer warps (4)   stage K_j (2-deep ring, freed when S_j completes) and V_j (2-deep ring, freed when
//                        P_j V_j completes) in the 128-byte-swizzled UMMA layout: the int8 state prefix arrives
//                        by TMA in a raw staging buffer and is dequantised from there exactly as materialize()
//                        rounds (bf16(q * s); fp16 scales: bf16(fp16(q * s))), the bf16 question prefix and own
//                        keys arrive by TMA directly; one visibility bit per key (padding, holes, segment ends)
//                        goes to a 4-deep mask ring
//   MMA warp (1 thread)  S_{j+1} = Q K_{j+1}^T into the other half of a double-buffered S in TMEM while the softmax
//                        works on S_j, then O += P_j V_j; Q and P are A operands in TMEM (shared memory then only
//                        streams K and V to the tensor core: its operand bandwidth is the limit), V is MN-major,
//                        O accumulates in TMEM
//   softmax warps (8)    warps 0-3 serve query tile 0 and warps 4-7 tile 1; warp w owns TMEM lane quarter w % 4, so
//                        one thread owns one query slot and all 128 keys of each block (no cross-warp exchange):
//                        causal and same-row masks on own keys, online softmax in the exp2 domain with a lazy
//                        rescale of O only when the max grows by more than 2^8, P (bf16) into TMEM; at the start each
//                        puts its slot's Q row into the tile's shared-memory operand, at the end O / l and the
//                        natural-log LSE
// Every mbarrier wait is bounded; a time-out ends the kernel with an error code, never a hang.
// Each slot's math does not depend on the other slots: outputs do not depend on row order.
#include <cudaTypedefs.h>

#include <string.h>

#include <type_traits>

#include "sm100.cuh"

namespace od {
namespace {
using namespace sm100;

constexpr int kSoftmaxWarps = 8;     // warps 0-3: query tile 0, warps 4-7: query tile 1 (lane quarter w % 4)
constexpr int kMmaWarp = 8;          // warp 8: TMEM allocation and the single MMA-issuing thread
constexpr int kProducerWarps = 4;    // warps 9-12: K/V blocks
constexpr int kProducer0 = 32 * (kSoftmaxWarps + 1);
constexpr int kProducers = 32 * kProducerWarps;
constexpr int kThreads = 32 * (kSoftmaxWarps + 1 + kProducerWarps);
constexpr int BM = 128;              // query slots per tile (one per TMEM lane)
constexpr int kMaxTiles = 2;         // query tiles per CTA (NT = 1 or 2), ping-ponged on the tensor core
constexpr int BN = 128;              // keys per block (one per producer thread)
constexpr int KS = 2;                // K ring depth
constexpr int VS = 2;                // V ring depth
constexpr int MS = 4;                // mask ring depth (a block's bits are rewritten only after both softmaxes)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;       // S of tile x at column x * BN (BN fp32); its P (bf16 pairs) overwrites the
                                     // first BN / 2 of those columns
constexpr uint32_t kTmemO = 2 * BN;  // O of tile x at column kTmemO + x * 128 (D <= 128 fp32)
constexpr int32_t kErrAttn = 0x5A0000;
static_assert(BN == kProducers, "one key of a block per producer thread");
static_assert(kTmemO + kMaxTiles * 128 <= kTmemCols, "TMEM columns");

template <int D, int NT>
struct Layout {
  static constexpr int ATOM = 128 * 128;             // 128 rows x 128 B: one 64-column swizzle atom of a tile
  static constexpr int TILE = ATOM * (D / 64);       // 128 rows x D bf16 (a Q tile, a K block or a V block)
  static constexpr int RD = NT == 1 ? 2 : 1;         // raw int8 staging depth (one query tile leaves room for 2)
  static constexpr int Q0 = 0;                       // NT query tiles (the A operand of S = Q K^T)
  static constexpr int K0 = Q0 + NT * TILE;
  static constexpr int V0 = K0 + KS * TILE;
  static constexpr int RAW0 = V0 + VS * TILE;        // RD x (int8 K block, int8 V block): BN rows x D bytes each
  static constexpr int MASK0 = RAW0 + RD * 2 * BN * D;   // MS x 4 words: bit k of word w = key 32 w + k visible
  static constexpr int BAR = MASK0 + MS * 16;        // mbarriers + TMEM holder + abort flag
  static constexpr int BYTES = BAR + 512 + 1024;     // + alignment slack
  static __host__ __device__ constexpr int Q(int x) { return Q0 + x * TILE; }
  static __host__ __device__ constexpr int K(int b) { return K0 + b * TILE; }
  static __host__ __device__ constexpr int V(int b) { return V0 + b * TILE; }
  static __host__ __device__ constexpr int RAWK(int r) { return RAW0 + r * 2 * BN * D; }
  static __host__ __device__ constexpr int RAWV(int r) { return RAWK(r) + BN * D; }
};
static_assert(Layout<128, 1>::BYTES <= 232448 && Layout<128, 2>::BYTES <= 232448, "shared memory");

struct Params {
  CUtensorMap map_ko, map_vo, map_kq, map_vq;   // bf16 (rows, Hkv*D) views of own / question K and V, 64x128 boxes
  CUtensorMap map_kp, map_vp;                   // (S*Hkv*T, D) views of the state prefix: int8 with D x 128 boxes,
                                                // or bf16 (materialised) with 64x128 boxes in the UMMA swizzle
  CUtensorMap map_q, map_o;                     // (R*t, Hq, D) views of q and o, boxes of 64 x rep x 128 / rep: one
                                                // box = 128 consecutive slots (token, head of the group) x 64 columns
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
  int64_t R, t, T, Lq;
  int Hq, Hkv, rep, tiles_per_group;
  int prefix_bf16;
  int nsplit;                                   // CTAs sharing one query tile's state prefix (grid z)
  int q_tma;                                    // the query tiles arrive by TMA and full output tiles leave by TMA
                                                // (map_q / map_o valid: rep divides 128)
  float* part_o;                                // nsplit > 1: per split, O / l (fp32, the layout of o) ...
  float* part_lse;                              // ... and the natural-log LSE (the layout of lse)
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

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// A producer thread's share of an int8 block: chunks c = pt + it * kProducers (16 bytes each, key c / (D / 16)).
template <int D>
struct Piece {
  static constexpr int N = BN * (D / 16) / kProducers;
};

// The scales of the thread's chunks, raw 16-bit patterns (nothing consumes them until the piece is converted, so
// the loads stay in flight meanwhile); keys past the segment get 0.
template <int D>
__device__ __forceinline__ void load_scales(uint32_t (&sc)[Piece<D>::N], int pt, const void* base, int p0,
                                            int p_hi) {
  constexpr int CPR = D / 16;
#pragma unroll
  for (int it = 0; it < Piece<D>::N; ++it) {
    const int p = p0 + (pt + it * kProducers) / CPR;
    sc[it] = p < p_hi ? static_cast<uint32_t>(__ldg(static_cast<const unsigned short*>(base) + p)) : 0u;
  }
}

// Dequantise a staged int8 block (row-major, D bytes per key) into a bf16 stage exactly as materialize() rounds.
template <typename TS, int D>
__device__ __forceinline__ void convert_piece(const uint8_t* raw, const uint32_t (&sc)[Piece<D>::N], uint8_t* dst,
                                              int pt) {
  constexpr int CPR = D / 16;
  constexpr int ATOM = Layout<D, 1>::ATOM;
#pragma unroll
  for (int it = 0; it < Piece<D>::N; ++it) {
    const int c = pt + it * kProducers;
    const int key = c / CPR, ch = c % CPR;
    const uint4 q = *reinterpret_cast<const uint4*>(raw + key * D + ch * 16);
    uint32_t w[8];
    if (std::is_same<TS, __nv_bfloat16>::value) {
      const uint32_t s2 = sc[it] | (sc[it] << 16);
      dequant4_bf16(q.x, s2, w[0], w[1]);
      dequant4_bf16(q.y, s2, w[2], w[3]);
      dequant4_bf16(q.z, s2, w[4], w[5]);
      dequant4_bf16(q.w, s2, w[6], w[7]);
    } else {
      // fp16 scales: bf16(fp16(q * s)) without conversion instructions. The byte q + 128 placed under the fp16
      // exponent of 1024 reads as 1024 + q + 128 (exact), minus 1152 gives q exactly; the packed fp16 multiply
      // rounds q * s once, as the reference's fp16 multiply does (q * s is exact in fp32); widening to fp32 is exact
      // and the bf16 pack rounds to nearest even.
      const uint32_t s2 = sc[it] | (sc[it] << 16);
      const __half2 sh = *reinterpret_cast<const __half2*>(&s2);
      const __half2 bias = __float2half2_rn(1152.0f);
      const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t u = words[b] ^ 0x80808080u;
        const uint32_t lo = __byte_perm(u, 0x64646464u, 0x4140), hi = __byte_perm(u, 0x64646464u, 0x4342);
        const __half2 qlo = __hsub2(*reinterpret_cast<const __half2*>(&lo), bias);
        const __half2 qhi = __hsub2(*reinterpret_cast<const __half2*>(&hi), bias);
        const float2 plo = __half22float2(__hmul2(qlo, sh)), phi = __half22float2(__hmul2(qhi, sh));
        w[2 * b] = pack_bf16(plo.x, plo.y);
        w[2 * b + 1] = pack_bf16(phi.x, phi.y);
      }
    }
    // the 16 int8 values of chunk ch are bf16 chunks 2ch and 2ch+1 of the row
    *reinterpret_cast<uint4*>(dst + swz(key, 2 * ch, ATOM)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(dst + swz(key, 2 * ch + 1, ATOM)) = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// Warp-uniform bounded wait (the softmax warps issue warp-collective TMEM accesses after it).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int32_t* err,
                                          int32_t code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, err, code));
}

template <typename TS, int D, int NT>
__global__ void __launch_bounds__(kThreads, 1) prefix_attn_kernel(const __grid_constant__ Params P) {
  using L = Layout<D, NT>;
  constexpr int RD = L::RD;
  constexpr int kCtaSlots = NT * BM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // pointer arithmetic on the shared array (not an integer cast) keeps the shared address space visible to the
  // compiler, so accesses compile to shared-memory instructions rather than generic ones
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* kfull = bars;                  // [KS] producers (+ TMA bytes) -> MMA
  uint64_t* kempty = kfull + KS;           // [KS] MMA (S_j of both tiles complete) -> producers
  uint64_t* vfull = kempty + KS;           // [VS] producers (+ TMA bytes) -> MMA
  uint64_t* vempty = vfull + VS;           // [VS] MMA (P_j V_j of both tiles complete) -> producers
  uint64_t* mfull = vempty + VS;           // [MS] producer warps (mask words written) -> softmax
  // s_full / p_full: per query tile (NT = 2), or per S buffer (NT = 1: S double-buffered in TMEM, buffer j & 1)
  uint64_t* s_full = mfull + MS;           // [2] MMA (S_j complete) -> softmax
  uint64_t* p_full = s_full + 2;           // [2] softmax (P_j in TMEM, O rescaled) -> MMA
  uint64_t* pv_done = p_full + 2;          // [NT] MMA (P_j V_j of the tile complete) -> softmax rescale, epilogue
  uint64_t* rawk_full = pv_done + NT;      // [RD] TMA (raw int8 K block) -> producers
  uint64_t* rawk_empty = rawk_full + RD;   // [RD] producers (raw K converted) -> the TMA-issuing producer
  uint64_t* rawv_full = rawk_empty + RD;   // [RD]
  uint64_t* rawv_empty = rawv_full + RD;   // [RD]
  uint64_t* q_full = rawv_empty + RD;      // softmax warps (the Q tiles in shared memory) -> MMA
  uint64_t* drain = q_full + 1;
  uint64_t* o_ready = drain + 1;           // [2] the tile's softmax threads (O rows staged) -> the TMA-store thread
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(o_ready + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  uint32_t* masks = reinterpret_cast<uint32_t*>(sm + L::MASK0);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x % P.tiles_per_group;
  const int grp = blockIdx.x / P.tiles_per_group;
  const int row0 = P.row_groups ? P.row_groups[2 * grp] : grp;
  const int nr = P.row_groups ? P.row_groups[2 * grp + 1] : 1;
  const int g = blockIdx.y, rep = P.rep;
  const int t = static_cast<int>(P.t);
  const int slots_row = t * rep;
  const int slots = nr * slots_row;
  const int s0 = tile * kCtaSlots;
  if (s0 >= slots) return;                            // uniform: before any barrier or allocation
  const int ntiles = NT == 2 && slots - s0 > BM ? 2 : 1;   // the second query tile only when it holds a slot
  const int split = blockIdx.z;

  if (tid == 0) {
    for (int b = 0; b < KS; ++b) {
      mbar_init(&kfull[b], kProducers);
      mbar_init(&kempty[b], 1);
    }
    for (int b = 0; b < VS; ++b) {
      mbar_init(&vfull[b], kProducers);
      mbar_init(&vempty[b], 1);
    }
    for (int b = 0; b < MS; ++b) mbar_init(&mfull[b], kProducerWarps);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&p_full[x], BM);
    }
    for (int x = 0; x < NT; ++x) {
      mbar_init(&pv_done[x], 1);
    }
    for (int r = 0; r < RD; ++r) {
      mbar_init(&rawk_full[r], 1);
      mbar_init(&rawk_empty[r], kProducers);
      mbar_init(&rawv_full[r], 1);
      mbar_init(&rawv_empty[r], kProducers);
    }
    mbar_init(q_full, P.q_tma ? 1 : 32 * 4 * NT);
    mbar_init(drain, 1);
    mbar_init(&o_ready[0], BM);
    mbar_init(&o_ready[1], BM);
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
  // with nsplit > 1 the state prefix's blocks are divided among the splits in contiguous runs and the last split
  // also takes the question prefix and the own keys
  int nb1 = 0, lo1 = 0, hi1 = 0, st = 0;
  const bool last_split = split == P.nsplit - 1;
  if (P.Kp) {
    st = P.row_state[row0];
    lo1 = P.p_lo ? P.p_lo[st] : 0;
    hi1 = P.p_hi ? P.p_hi[st] : static_cast<int>(P.T);
    const int all = hi1 > lo1 ? (hi1 - lo1 + BN - 1) / BN : 0;
    const int per = (all + P.nsplit - 1) / P.nsplit;
    const int b0 = min(all, split * per), b1 = min(all, b0 + per);
    nb1 = b1 - b0;
    lo1 += b0 * BN;
    hi1 = min(hi1, lo1 + nb1 * BN);
  }
  int nb2 = 0, n2 = 0, qr = 0;
  if (P.Kq && last_split) {
    qr = P.row_q[row0];
    n2 = P.q_len[qr];
    nb2 = (n2 + BN - 1) / BN;
  }
  // own keys, flattened (row a, token j) -> a * t + j; a single long row only needs keys up to the CTA's last token
  int own_begin = 0, own_end = last_split ? nr * t : 0;
  if (nr == 1 && last_split) {
    const int lo = P.own_lo ? P.own_lo[row0] : 0;
    const int last_tok = min(t - 1, (min(slots, s0 + kCtaSlots) - 1) / rep);
    own_begin = (lo / BN) * BN;
    own_end = last_tok + 1;
  }
  const int nb3 = own_end > own_begin ? (own_end - own_begin + BN - 1) / BN : 0;
  const int nblk = nb1 + nb2 + nb3;

  if (warp > kMmaWarp) {
    // ================================================================== producers: K/V blocks
    const int pt = tid - kProducer0, pw = pt >> 5;
    if (P.q_tma && pt == 0 && nblk > 0) {
      // the CTA's query tiles: tile x = slots s0 + x BM .. + BM - 1 of the group = tokens row0 t + (s0 + x BM) / rep ..
      // (all heads of the GQA group per token); tokens past the last row read as zero, slots past the group's last
      // read the next group's rows (finite; never stored)
      mbar_arrive_expect_tx(q_full, ntiles * L::TILE);
      for (int x = 0; x < ntiles; ++x)
#pragma unroll
        for (int h = 0; h < D / 64; ++h)
          tma_load_3d(sm + L::Q(x) + h * L::ATOM, &P.map_q, q_full, h * 64, g * rep, row0 * t + (s0 + x * BM) / rep);
    }
    const TS* ks1 = nullptr;
    const TS* vs1 = nullptr;
    const uint8_t* pm1 = nullptr;
    int prow = 0;                                     // row of key 0 in the (S*Hkv*T, D) int8 views
    if (P.Kp) {
      const int64_t base = (static_cast<int64_t>(st) * P.Hkv + g) * P.T;
      prow = static_cast<int>(base);
      if (!P.prefix_bf16) {
        ks1 = static_cast<const TS*>(P.ksc) + base;
        vs1 = static_cast<const TS*>(P.vsc) + base;
      }
      pm1 = P.pmask ? P.pmask + static_cast<int64_t>(st) * P.T : nullptr;
    }
    uint32_t skc[Piece<D>::N], svc[Piece<D>::N];     // scales of the next int8 K / V piece to convert
    if (nb1 > 0 && !P.prefix_bf16) {
      load_scales<D>(skc, pt, ks1, lo1, hi1);
      load_scales<D>(svc, pt, vs1, lo1, hi1);
      if (pt == 0) {                                  // the first RD raw blocks in flight
        for (int r = 0; r < RD && r < nb1; ++r) {
          mbar_arrive_expect_tx(&rawk_full[r], BN * D);
          tma_load_2d(sm + L::RAWK(r), &P.map_kp, &rawk_full[r], 0, prow + lo1 + r * BN);
          mbar_arrive_expect_tx(&rawv_full[r], BN * D);
          tma_load_2d(sm + L::RAWV(r), &P.map_vp, &rawv_full[r], 0, prow + lo1 + r * BN);
        }
      }
    }
    for (int j = 0; j < nblk; ++j) {
      const bool pre = j < nb1;                       // state prefix block
      const bool i8 = pre && !P.prefix_bf16;          // ... dequantised here
      const bool q_seg = !pre && j < nb1 + nb2;
      const int k0 = pre ? lo1 + j * BN : q_seg ? (j - nb1) * BN : own_begin + (j - nb1 - nb2) * BN;
      // ---- K_j (a mask slot, written below, is reused 4 blocks later: by then this producer has passed the K stage
      // wait of block j+4, which follows S of block j+2 in both tiles and so both softmaxes of block j+1)
      const int bk = j % KS;
      if (j >= KS && !mbar_wait(&kempty[bk], ((j / KS) - 1) & 1, abort_flag, P.err, kErrAttn | 1)) break;
      uint8_t* sK = sm + L::K(bk);
      if (i8) {
        const int r = j % RD;
        if (!mbar_wait(&rawk_full[r], (j / RD) & 1, abort_flag, P.err, kErrAttn | 13)) break;
        convert_piece<TS, D>(sm + L::RAWK(r), skc, sK, pt);
        mbar_arrive(&rawk_empty[r]);
        if (j + 1 < nb1) load_scales<D>(skc, pt, ks1, k0 + BN, hi1);
        if (j + RD < nb1 && pt == 0) {                // refill the staging slot once every thread has converted it
          if (!mbar_wait(&rawk_empty[r], (j / RD) & 1, abort_flag, P.err, kErrAttn | 14)) break;
          mbar_arrive_expect_tx(&rawk_full[r], BN * D);
          tma_load_2d(sm + L::RAWK(r), &P.map_kp, &rawk_full[r], 0, prow + k0 + RD * BN);
        }
        fence_proxy_async_smem();
        mbar_arrive(&kfull[bk]);
      } else if (pt == 0) {
        const CUtensorMap* mk = pre ? &P.map_kp : q_seg ? &P.map_kq : &P.map_ko;
        const int y = pre ? prow + k0 : (q_seg ? qr * static_cast<int>(P.Lq) : row0 * t) + k0;
        const int x0 = pre ? 0 : g * D;
        mbar_arrive_expect_tx(&kfull[bk], L::TILE);
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(sK + h * L::ATOM, mk, &kfull[bk], x0 + h * 64, y);
      } else {
        mbar_arrive(&kfull[bk]);
      }
      // ---- the block's visibility bits, after K_j is on its way (their global loads stay off the K path)
      bool vis;
      {
        const int idx = k0 + pt;
        if (pre) {
          vis = idx < hi1 && (!pm1 || pm1[idx]);
        } else if (q_seg) {
          vis = idx < n2;
        } else {
          const int a = idx / t, jj = idx - a * t;
          const int r = row0 + a;
          vis = idx < own_end && a < nr && jj >= (P.own_lo ? P.own_lo[r] : 0) && jj < (P.own_hi ? P.own_hi[r] : t);
        }
      }
      const uint32_t word = __ballot_sync(0xffffffffu, vis);
      if (lane == 0) {
        masks[4 * (j % MS) + pw] = word;
        mbar_arrive(&mfull[j % MS]);
      }
      // ---- V_j
      const int bv = j % VS;
      if (j >= VS && !mbar_wait(&vempty[bv], ((j / VS) - 1) & 1, abort_flag, P.err, kErrAttn | 2)) break;
      uint8_t* sV = sm + L::V(bv);
      if (i8) {
        const int r = j % RD;
        if (!mbar_wait(&rawv_full[r], (j / RD) & 1, abort_flag, P.err, kErrAttn | 15)) break;
        convert_piece<TS, D>(sm + L::RAWV(r), svc, sV, pt);
        mbar_arrive(&rawv_empty[r]);
        if (j + 1 < nb1) load_scales<D>(svc, pt, vs1, k0 + BN, hi1);
        if (j + RD < nb1 && pt == 0) {
          if (!mbar_wait(&rawv_empty[r], (j / RD) & 1, abort_flag, P.err, kErrAttn | 16)) break;
          mbar_arrive_expect_tx(&rawv_full[r], BN * D);
          tma_load_2d(sm + L::RAWV(r), &P.map_vp, &rawv_full[r], 0, prow + k0 + RD * BN);
        }
        fence_proxy_async_smem();
        mbar_arrive(&vfull[bv]);
      } else if (pt == 0) {
        const CUtensorMap* mv = pre ? &P.map_vp : q_seg ? &P.map_vq : &P.map_vo;
        const int y = pre ? prow + k0 : (q_seg ? qr * static_cast<int>(P.Lq) : row0 * t) + k0;
        const int x0 = pre ? 0 : g * D;
        mbar_arrive_expect_tx(&vfull[bv], L::TILE);
#pragma unroll
        for (int h = 0; h < D / 64; ++h) tma_load_2d(sV + h * L::ATOM, mv, &vfull[bv], x0 + h * 64, y);
      } else {
        mbar_arrive(&vfull[bv]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ================================================================== MMA issue (one thread)
    // Per block j and tile x: S_x(j) = Q_x K_j^T into the tile's S columns, then (once the tile's softmax has
    // written P_x(j) over them) O_x += P_x(j) V_j. P aliases S, so S_x(j+1) is issued only after P_x(j) V_j has
    // completed; the other tile's MMAs fill the tensor core meanwhile (A: P V, S; then B: P V, S).
    // One query tile (NT = 1): the second tile's S columns hold a second S buffer, so S(j+1) is computed while the
    // softmax works on block j and the softmax runs block after block; S(j+2) follows P(j) V(j) into buffer j & 1.
    if constexpr (NT == 1) {
      if (lane == 0 && nblk > 0) {
        constexpr uint32_t idesc_s = idesc_bf16(BM, BN, false);
        constexpr uint32_t idesc_o = idesc_bf16(BM, D, true);
        // descriptors computed once; each MMA then costs its issuing thread one add and the instruction
        static_assert(KS == 2 && VS == 2, "two stages");
        const uint64_t qd = desc_sw128(smem_u32(sm + L::Q(0)), 16, 1024);
        const uint64_t kd0 = desc_sw128(smem_u32(sm + L::K(0)), 16, 1024);
        const uint64_t kd1 = desc_sw128(smem_u32(sm + L::K(1)), 16, 1024);
        const uint64_t vd0 = desc_sw128(smem_u32(sm + L::V(0)), L::ATOM, 1024);
        const uint64_t vd1 = desc_sw128(smem_u32(sm + L::V(1)), L::ATOM, 1024);
        auto issue_s = [&](int j) {
          const uint64_t kd = (j % KS) ? kd1 : kd0;
          const uint32_t dS = tmem + kTmemS + (j & 1) * BN;
          mma_f16(dS, qd, kd, idesc_s, 0u);
#pragma unroll
          for (int k = 1; k < D / 16; ++k) {
            const uint32_t off = (k >> 2) * L::ATOM + (k & 3) * 32;
            mma_f16_accum(dS, desc_advance(qd, off), desc_advance(kd, off), idesc_s);
          }
          mma_commit(&s_full[j & 1]);
          mma_commit(&kempty[j % KS]);
        };
        bool live = mbar_wait(q_full, 0, abort_flag, P.err, kErrAttn | 17);
        for (int j = 0; j < 2 && j < nblk && live; ++j) {
          live = mbar_wait(&kfull[j % KS], (j / KS) & 1, abort_flag, P.err, kErrAttn | 3);
          if (live) {
            tc_fence_after();
            issue_s(j);
          }
        }
        for (int j = 0; j < nblk && live; ++j) {
          if (!mbar_wait(&vfull[j % VS], (j / VS) & 1, abort_flag, P.err, kErrAttn | 5) ||
              !mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_flag, P.err, kErrAttn | 6))
            break;
          tc_fence_after();
          const uint64_t vd = (j % VS) ? vd1 : vd0;
          const uint32_t aP = tmem + kTmemS + (j & 1) * BN;
          mma_f16_ts(tmem + kTmemO, aP, vd, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 1; kk < BN / 16; ++kk)
            mma_f16_ts_accum(tmem + kTmemO, aP + kk * 8, desc_advance(vd, kk * 16 * 128), idesc_o);
          mma_commit(&pv_done[0]);
          mma_commit(&vempty[j % VS]);
          if (j + 2 < nblk) {
            if (!mbar_wait(&kfull[(j + 2) % KS], ((j + 2) / KS) & 1, abort_flag, P.err, kErrAttn | 4)) break;
            tc_fence_after();
            issue_s(j + 2);                         // in issue order behind the P.V that reads buffer j & 1
          }
        }
        mma_commit(drain);
        const long long c0 = clock64();
        while (!mbar_try_wait(drain, 0) && clock64() - c0 < kWaitLimitCycles) {
        }
      }
    } else if (lane == 0 && nblk > 0) {
      constexpr uint32_t idesc_s = idesc_bf16(BM, BN, false);
      constexpr uint32_t idesc_o = idesc_bf16(BM, D, true);
      // descriptors computed once; each MMA then costs its issuing thread one add and the instruction
      static_assert(KS == 2 && VS == 2, "two stages");
      const uint64_t qd0 = desc_sw128(smem_u32(sm + L::Q(0)), 16, 1024);
      const uint64_t qd1 = desc_sw128(smem_u32(sm + L::Q(NT - 1)), 16, 1024);
      const uint64_t kd0 = desc_sw128(smem_u32(sm + L::K(0)), 16, 1024);
      const uint64_t kd1 = desc_sw128(smem_u32(sm + L::K(1)), 16, 1024);
      const uint64_t vd0 = desc_sw128(smem_u32(sm + L::V(0)), L::ATOM, 1024);
      const uint64_t vd1 = desc_sw128(smem_u32(sm + L::V(1)), L::ATOM, 1024);
      auto issue_s = [&](int x, int j) {
        const uint64_t qd = x ? qd1 : qd0, kd = (j % KS) ? kd1 : kd0;
        const uint32_t dS = tmem + kTmemS + x * BN;
        mma_f16(dS, qd, kd, idesc_s, 0u);
#pragma unroll
        for (int k = 1; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * L::ATOM + (k & 3) * 32;
          mma_f16_accum(dS, desc_advance(qd, off), desc_advance(kd, off), idesc_s);
        }
        mma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {
        const uint64_t vd = (j % VS) ? vd1 : vd0;
        const uint32_t dO = tmem + kTmemO + x * 128, aP = tmem + kTmemS + x * BN;
        mma_f16_ts(dO, aP, vd, idesc_o, j > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 1; kk < BN / 16; ++kk) mma_f16_ts_accum(dO, aP + kk * 8, desc_advance(vd, kk * 16 * 128), idesc_o);
        mma_commit(&pv_done[x]);
      };
      bool live = mbar_wait(q_full, 0, abort_flag, P.err, kErrAttn | 17) &&
                  mbar_wait(&kfull[0], 0, abort_flag, P.err, kErrAttn | 3);
      if (live) {
        tc_fence_after();
        for (int x = 0; x < ntiles; ++x) issue_s(x, 0);
        mma_commit(&kempty[0]);
      }
      for (int j = 0; j < nblk && live; ++j) {
        const bool more = j + 1 < nblk;
        if (!mbar_wait(&vfull[j % VS], (j / VS) & 1, abort_flag, P.err, kErrAttn | 5)) break;
        if (more && !mbar_wait(&kfull[(j + 1) % KS], ((j + 1) / KS) & 1, abort_flag, P.err, kErrAttn | 4)) break;
        for (int x = 0; x < ntiles && live; ++x) {
          if (!mbar_wait(&p_full[x], j & 1, abort_flag, P.err, kErrAttn | 6)) {
            live = false;
            break;
          }
          tc_fence_after();
          issue_pv(x, j);
          if (x == ntiles - 1) mma_commit(&vempty[j % VS]);
          if (more) {
            // S_x(j+1) overwrites the columns P_x(j) V_j reads: the tensor core executes one thread's MMAs in issue
            // order, so it follows right behind without a wait
            issue_s(x, j + 1);
            if (x == ntiles - 1) mma_commit(&kempty[(j + 1) % KS]);
          }
        }
      }
      // every MMA issued here has completed before TMEM is released (immediate unless aborted)
      mma_commit(drain);
      const long long c0 = clock64();
      while (!mbar_try_wait(drain, 0) && clock64() - c0 < kWaitLimitCycles) {
      }
    }
  } else {
    // ================================================================== softmax (tile x, lane quarter q4)
    const int q4 = warp & 3, x = warp >> 2;
    const int tt = 32 * q4 + lane;                    // slot of the tile = TMEM lane
    const int slot = s0 + x * BM + tt;
    const bool my_valid = slot < slots;
    const int a_my = my_valid ? slot / slots_row : 0;
    const int i_my = my_valid ? (slot % slots_row) / rep : 0;
    const int hh_my = slot % rep;
    const uint32_t lane_off = static_cast<uint32_t>(32 * q4) << 16;
    const uint32_t tS0 = tmem + lane_off + kTmemS + x * BN;
    const uint32_t tO = tmem + lane_off + kTmemO + x * 128;
    const float scale = P.scale_log2;
    if (x < NT && !P.q_tma) {
      // the warp's 32 Q rows (tile rows 32 q4 ..) into the tile's shared-memory A operand (128-byte swizzled,
      // K-major), row by row across the warp: each load instruction reads 32 / CPR whole rows (contiguous 16-byte
      // chunks), so every fetched line is used at once. (One thread per row, 16 strided loads each, re-fetched the
      // lines from L2 up to 8 times once the small L1 beside ~200 KB of shared memory had evicted them.)
      // Slots past the group's last are zero.
      uint8_t* dq = sm + L::Q(x);
      constexpr int CPR = D / 8;                      // 16-byte chunks per row
      constexpr int RPI = 32 / CPR;                   // rows per instruction
      constexpr int HALF = CPR / 2;                   // loads in flight per batch
      const int ch = lane % CPR;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint4 val[HALF];
#pragma unroll
        for (int it = 0; it < HALF; ++it) {
          const int sl = s0 + x * BM + 32 * q4 + (b * HALF + it) * RPI + lane / CPR;
          val[it] = make_uint4(0, 0, 0, 0);
          if (sl < slots) {
            const int a = sl / slots_row, i = (sl % slots_row) / rep, hh = sl % rep;
            val[it] = __ldg(reinterpret_cast<const uint4*>(
                              P.q + ((static_cast<int64_t>(row0 + a) * t + i) * P.Hq + g * rep + hh) * D) + ch);
          }
        }
#pragma unroll
        for (int it = 0; it < HALF; ++it)
          *reinterpret_cast<uint4*>(dq + swz(32 * q4 + (b * HALF + it) * RPI + lane / CPR, ch, L::ATOM)) = val[it];
      }
      fence_proxy_async_smem();
      mbar_arrive(q_full);
    }
    const bool active = x < ntiles;                   // warp-uniform
    float m_used = -INFINITY, l_sum = 0.f;
    bool live = true;
    for (int j = 0; j < nblk && active; ++j) {
      const int sb = NT == 1 ? (j & 1) : x;          // S buffer of this block
      if (!warp_wait(&s_full[sb], NT == 1 ? (j >> 1) & 1 : j & 1, abort_flag, P.err, kErrAttn | 7) ||
          !warp_wait(&mfull[j % MS], (j / MS) & 1, abort_flag, P.err, kErrAttn | 8)) {
        live = false;
        break;
      }
      const uint32_t tS = NT == 1 ? tS0 + (j & 1) * BN : tS0;
      tc_fence_after();
      uint32_t mw[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) mw[w] = masks[4 * (j % MS) + w];
      // own keys visible to this slot form one range of the flattened (row, token) index: its own row's tokens up
      // to its own position; in block-local key numbers: [vis_lo, vis_hi]
      int vis_lo = -(1 << 30), vis_hi = 1 << 30;
      if (j >= nb1 + nb2) {
        const int key0 = own_begin + (j - nb1 - nb2) * BN;
        vis_lo = a_my * t - key0;
        vis_hi = a_my * t + i_my - key0;
      }
      const bool fast = __all_sync(0xffffffffu, (mw[0] & mw[1] & mw[2] & mw[3]) == 0xffffffffu && vis_lo <= 0 &&
                                                    vis_hi >= BN - 1);
      // a 32-key chunk's scores with the invisible keys at -inf
      auto mask_chunk = [&](uint32_t (&c)[32], int ci) {
        if (!fast) {
          const uint32_t w = ci == 0 ? mw[0] : ci == 1 ? mw[1] : ci == 2 ? mw[2] : mw[3];
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (!((w >> k) & 1u) || k + 32 * ci < vis_lo || k + 32 * ci > vis_hi) c[k] = __float_as_uint(-INFINITY);
        }
      };
      // P = 2^(s * scale - m) in bf16 over the S columns (P chunk c lands on columns 16c..16c+15, which hold S chunk
      // c / 2: already read), the row sum in fp32; returns the block's row max (scaled). One 32-key chunk of scores
      // in registers at a time (the kernel's 13 warps cap a thread at 128 registers).
      float2 acc[2];
      auto p_pass = [&](float m) -> float {
        const bool none = m == -INFINITY;              // no visible key so far: every weight is 0
        const float2 sc2 = make_float2(scale, scale), nm2 = make_float2(-m, -m);
        acc[0] = acc[1] = make_float2(0.f, 0.f);
        float mq[2] = {-INFINITY, -INFINITY};
#pragma unroll 1
        for (int ci = 0; ci < 4; ++ci) {
          uint32_t cc[32];
          tmem_ld_32x32b_x32(tS + 32 * ci, cc);
          tmem_ld_wait();
          mask_chunk(cc, ci);
          uint32_t pw[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float e0 = __uint_as_float(cc[2 * k]), e1 = __uint_as_float(cc[2 * k + 1]);
            mq[k & 1] = fmax3(mq[k & 1], e0, e1);
            if (none) {
              pw[k] = 0u;
            } else {
              const float2 y = __ffma2_rn(make_float2(e0, e1), sc2, nm2);
              const float2 pp = make_float2(ex2_approx(y.x), ex2_approx(y.y));
              acc[k & 1] = __fadd2_rn(acc[k & 1], pp);
              pw[k] = pack_bf16(pp.x, pp.y);
            }
          }
          tmem_st_32x32b_x16(tS + 16 * ci, pw);
        }
        return fmaxf(mq[0], mq[1]) * scale;
      };
      // O_x may be rescaled once P_x(j-1) V_{j-1} has completed: with two tiles it did before S_x(j) was issued;
      // with one (S double-buffered) the softmax waits for it here
      auto rescale_o = [&](float alpha, bool resc) -> bool {
        if (__any_sync(0xffffffffu, resc)) {
          if (NT == 1 && j > 0 && !warp_wait(&pv_done[0], (j - 1) & 1, abort_flag, P.err, kErrAttn | 18))
            return false;
          tc_fence_after();
#pragma unroll 1
          for (int dc = 0; dc < D / 32; ++dc) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(tO + dc * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st_32x32b_x32(tO + dc * 32, o);
          }
        }
        return true;
      };
      if (__any_sync(0xffffffffu, m_used == -INFINITY)) {
        // a lane has no running max yet: the block's row max first (a separate pass over S), then P
        uint32_t ca[32], cb[32];
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld_32x32b_x32(tS + 64 * half, ca);
          tmem_ld_32x32b_x32(tS + 64 * half + 32, cb);
          tmem_ld_wait();
          mask_chunk(ca, 2 * half);
          mask_chunk(cb, 2 * half + 1);
#pragma unroll
          for (int k = 0; k < 32; k += 4) {
            mq[0] = fmax3(mq[0], __uint_as_float(ca[k]), __uint_as_float(ca[k + 1]));
            mq[1] = fmax3(mq[1], __uint_as_float(ca[k + 2]), __uint_as_float(ca[k + 3]));
            mq[2] = fmax3(mq[2], __uint_as_float(cb[k]), __uint_as_float(cb[k + 1]));
            mq[3] = fmax3(mq[3], __uint_as_float(cb[k + 2]), __uint_as_float(cb[k + 3]));
          }
        }
        const float mb = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale;
        float alpha = 1.f;
        bool resc = false;
        if (m_used == -INFINITY) {
          m_used = mb;                                 // nothing accumulated yet: O and l are 0
        } else if (mb > m_used + 8.f) {
          alpha = ex2_approx(m_used - mb);
          l_sum *= alpha;
          m_used = mb;
          resc = true;
        }
        if (!rescale_o(alpha, resc)) {
          live = false;
          break;
        }
        p_pass(m_used);
      } else {
        // speculative: P against the running max; kept unless the block's max exceeds it by more than 2^8 (lazy
        // rescale), in which case O and l are rescaled and P is recomputed (the overwritten P never reached the MMA)
        const float mb = p_pass(m_used);
        const bool redo = mb > m_used + 8.f;
        if (__any_sync(0xffffffffu, redo)) {
          float alpha = 1.f;
          if (redo) {
            alpha = ex2_approx(m_used - mb);
            l_sum *= alpha;
            m_used = mb;
          }
          if (!rescale_o(alpha, redo)) {
            live = false;
            break;
          }
          p_pass(m_used);
        }
      }
      l_sum += (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // ---- epilogue: O / l, natural-log LSE (nothing is written after a time-out; the error word says why).
    // TMEM loads are warp-collective: every lane loads, valid slots store.
    if (active) {
      if (live && nblk > 0) live = warp_wait(&pv_done[x], (nblk - 1) & 1, abort_flag, P.err, kErrAttn | 11);
      if (live) {
        tc_fence_after();
        const float inv = l_sum > 0.f ? 1.0f / l_sum : 0.f;
        const int64_t orow = ((static_cast<int64_t>(row0 + a_my) * t + i_my) * P.Hq + g * rep + hh_my) * D;
        const int64_t lrow = (static_cast<int64_t>(row0 + a_my) * P.Hq + g * rep + hh_my) * t + i_my;
        const float lse_v = l_sum > 0.f ? (m_used + log2f(l_sum)) * 0.6931471805599453f : -INFINITY;
        // one split: bf16 O / l (and the LSE); several: this split's fp32 O / l and LSE, merged by od_attn_merge
        const int64_t n_l = P.R * P.t * P.Hq, n_o = n_l * D;
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t o[32];
          if (nblk > 0) {
            tmem_ld_32x32b_x32(tO + dc * 32, o);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = 0u;
          }
          if (my_valid) {
            if (P.nsplit > 1) {
              float4* dst = reinterpret_cast<float4*>(P.part_o + split * n_o + orow + dc * 32);
#pragma unroll
              for (int k = 0; k < 8; ++k)
                dst[k] = make_float4(__uint_as_float(o[4 * k]) * inv, __uint_as_float(o[4 * k + 1]) * inv,
                                     __uint_as_float(o[4 * k + 2]) * inv, __uint_as_float(o[4 * k + 3]) * inv);
            } else {
              // bf16 O / l into this slot's row of the tile's Q buffer (free: every MMA of the tile has completed),
              // in the same swizzled layout; the warp stores its 32 rows below, whole rows per instruction
              uint32_t w[16];
#pragma unroll
              for (int k = 0; k < 16; ++k)
                w[k] = pack_bf16(__uint_as_float(o[2 * k]) * inv, __uint_as_float(o[2 * k + 1]) * inv);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                *reinterpret_cast<uint4*>(sm + L::Q(x) + swz(tt, dc * 4 + k, L::ATOM)) =
                    make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
            }
          }
        }
        if (P.nsplit == 1 && P.q_tma && s0 + x * BM + BM <= slots) {
          // a full tile (every slot in the group): one TMA store per 64 columns once all 128 rows are staged
          fence_proxy_async_smem();
          mbar_arrive(&o_ready[x]);
          if (q4 == 0 && lane == 0 && mbar_wait(&o_ready[x], 0, abort_flag, P.err, kErrAttn | 19)) {
#pragma unroll
            for (int h = 0; h < D / 64; ++h)
              tma_store_3d(&P.map_o, sm + L::Q(x) + h * L::ATOM, h * 64, g * rep, row0 * t + (s0 + x * BM) / rep);
            tma_store_commit();
            tma_store_wait_read();
          }
        } else if (P.nsplit == 1) {
          __syncwarp();
          constexpr int CPR = D / 8, RPI = 32 / CPR;
          const int ch = lane % CPR;
#pragma unroll 4
          for (int it = 0; it < CPR; ++it) {
            const int rr = 32 * q4 + it * RPI + lane / CPR;
            const int sl = s0 + x * BM + rr;
            if (sl < slots) {
              const int a = sl / slots_row, i = (sl % slots_row) / rep, hh = sl % rep;
              reinterpret_cast<uint4*>(P.o + ((static_cast<int64_t>(row0 + a) * t + i) * P.Hq + g * rep + hh) * D)[ch] =
                  *reinterpret_cast<const uint4*>(sm + L::Q(x) + swz(rr, ch, L::ATOM));
            }
          }
        }
        if (my_valid) {
          if (P.nsplit > 1)
            P.part_lse[split * n_l + lrow] = lse_v;
          else if (P.lse)
            P.lse[lrow] = lse_v;
        }
      }
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

// (rows, cols) bf16 row-major view tiled into 64-column x BN-row boxes with the 128-byte swizzle of the UMMA layout
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

// (rows, Hq, D) bf16 view (q or o: token-major, heads, head_dim) tiled into 64 x rep x (BM / rep) boxes with the
// 128-byte swizzle: a box is BM consecutive (token, head) rows of 128 bytes, the UMMA layout of a query tile
int make_map_slots(CUtensorMap* map, const void* base, uint64_t D, uint64_t H, uint64_t rows, int rep) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {D, H, rows};
  cuuint64_t strides[2] = {D * 2, H * D * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(rep), static_cast<cuuint32_t>(BM / rep)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled (slots) failed (%d)", static_cast<int>(r));
  return OD_OK;
}

// (rows, D) int8 row-major view tiled into D x BN boxes, no swizzle (the producers read it row by row)
int make_map_i8(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return fail(OD_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(cols), static_cast<cuuint32_t>(BN)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OD_ECUDA, "cuTensorMapEncodeTiled (int8) failed (%d)", static_cast<int>(r));
  return OD_OK;
}

template <typename TS, int D, int NT>
int launch_attn(const Params& P, dim3 grid, cudaStream_t st) {
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    OD_CUDA_TRY(cudaFuncSetAttribute(prefix_attn_kernel<TS, D, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Layout<D, NT>::BYTES));
    attr[dev] = true;
  }
  prefix_attn_kernel<TS, D, NT><<<grid, kThreads, Layout<D, NT>::BYTES, st>>>(P);
  OD_LAUNCH_CHECK();
  return ok();
}

// The splits of a query row merged exactly by log-sum-exp (the Hydragen merge of prefix_attn._split_attention):
// O = sum_s w_s O_s / sum_s w_s, w_s = exp(lse_s - max lse), LSE = max lse + log sum_s w_s. One warp per output
// row (row, token, head), D / 32 elements per lane. When the device error word is set (a split gave up a bounded
// wait and may have left its partials unwritten, so the workspace can hold an earlier call's values), every output
// is NaN instead of a plausible mix.
template <int D>
__global__ void __launch_bounds__(256) attn_merge_kernel(const float* __restrict__ part_o,
                                                         const float* __restrict__ part_lse, int nsplit,
                                                         int64_t n_rows, int t, int Hq, __nv_bfloat16* __restrict__ o,
                                                         float* __restrict__ lse, const int32_t* __restrict__ err) {
  constexpr int E = D / 32;
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int64_t h = row % Hq, ri = row / Hq;
  const int64_t lrow = ((ri / t) * Hq + h) * t + ri % t;
  if (*reinterpret_cast<const volatile int32_t*>(err) != 0) {
    __nv_bfloat16* dst = o + row * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(NAN, NAN);
    if (lse && lane == 0) lse[lrow] = NAN;
    return;
  }
  float m = -INFINITY;
  for (int sp = 0; sp < nsplit; ++sp) m = fmaxf(m, __ldg(part_lse + sp * n_rows + lrow));
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  float wsum = 0.f;
  if (m != -INFINITY) {
    for (int sp = 0; sp < nsplit; ++sp) {
      const float w = expf(__ldg(part_lse + sp * n_rows + lrow) - m);
      wsum += w;
      const float* src = part_o + (sp * n_rows + row) * D + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] = fmaf(w, __ldg(src + e), acc[e]);
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  __nv_bfloat16* dst = o + row * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(acc[e] * inv, acc[e + 1] * inv);
  if (lse && lane == 0) lse[lrow] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
}

// Splits of the state prefix: the count minimising (waves of CTAs) x (blocks per CTA + 2 blocks of fixed cost);
// 1 when the query tiles alone fill the GPU.
int plan_splits(int64_t ctas, int64_t prefix_blocks, int num_sms) {
  if (ctas <= 0 || prefix_blocks < 4 || num_sms <= 0) return 1;
  int best = 1;
  double best_t = 1e300;
  for (int n = 1; n <= 8 && n <= prefix_blocks / 2; ++n) {
    const double waves = static_cast<double>((ctas * n + num_sms - 1) / num_sms);
    const double tm = waves * (static_cast<double>((prefix_blocks + n - 1) / n) + 2.0);
    if (tm < best_t * 0.97) {
      best_t = tm;
      best = n;
    }
  }
  return best;
}

int64_t group_slots(const od_attn_dims& d) {
  const int64_t rows = d.max_group_rows > 0 ? d.max_group_rows : 1;
  return rows * d.t * (d.Hq / (d.Hkv > 0 ? d.Hkv : 1));
}

}  // namespace
}  // namespace od

using namespace od;

extern "C" int od_prefix_attn(const void* q, const void* Kp, const void* Vp, const void* ksc, const void* vsc,
                              const int32_t* row_state, const int32_t* p_lo, const int32_t* p_hi, const uint8_t* pmask,
                              const void* Kq, const void* Vq, const int32_t* row_q, const int32_t* q_len,
                              const void* k_own, const void* v_own, const int32_t* own_lo, const int32_t* own_hi,
                              const int32_t* row_groups, void* o, float* lse, od_attn_dims dims, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  OD_REQUIRE(dims.D == 64 || dims.D == 128, "od_prefix_attn: head_dim %d not in {64, 128}", dims.D);
  OD_REQUIRE(dims.Hq > 0 && dims.Hkv > 0 && dims.Hq % dims.Hkv == 0, "od_prefix_attn: bad head counts");
  const int rep = dims.Hq / dims.Hkv;
  OD_REQUIRE(dims.R >= 0 && dims.t >= 0 && dims.t < (1 << 24), "od_prefix_attn: bad R/t");
  OD_REQUIRE(!row_groups || dims.G >= 0, "od_prefix_attn: bad row groups");
  // an empty problem needs no buffers (empty tensors may carry null pointers), no workspace and no launch
  if ((row_groups ? dims.G : dims.R) == 0 || dims.t == 0) return ok();
  OD_REQUIRE(q && k_own && v_own && o, "od_prefix_attn: null pointer");
  const bool pbf16 = dims.prefix_bf16 != 0;
  OD_REQUIRE(!Kp || (Vp && (pbf16 || (ksc && vsc)) && row_state && dims.S > 0 && dims.T > 0 && dims.T < (1 << 30)),
             "od_prefix_attn: the state prefix needs Vp, row_state, S, T (and ksc/vsc when int8)");
  OD_REQUIRE(!Kp || pbf16 || dims.scale_dtype == OD_BF16 || dims.scale_dtype == OD_F16, "od_prefix_attn: scale dtype");
  OD_REQUIRE(!Kq || (Vq && row_q && q_len && dims.NQ > 0 && dims.Lq > 0), "od_prefix_attn: bad question prefix");
  OD_REQUIRE(aligned16(q) && aligned16(k_own) && aligned16(v_own) && aligned16(o) &&
                 (!Kp || (aligned16(Kp) && aligned16(Vp))) && (!Kq || (aligned16(Kq) && aligned16(Vq))),
             "od_prefix_attn: tensors must be 16-byte aligned");
  const int64_t G = row_groups ? dims.G : dims.R;
  const int64_t max_rows = row_groups ? dims.max_group_rows : 1;
  OD_REQUIRE(G >= 0 && max_rows >= 1, "od_prefix_attn: bad row groups");
  OD_REQUIRE(max_rows == 1 || max_rows * dims.t * rep <= kMaxTiles * BM,
             "od_prefix_attn: a group of several rows must fit one CTA's %d slots (rows %lld x t %lld x rep %d)",
             kMaxTiles * BM, (long long)max_rows, (long long)dims.t, rep);
  const int64_t gslots = max_rows * dims.t * rep;
  const int NT = gslots <= BM ? 1 : 2;                // one query tile per CTA frees room for deeper int8 staging
  const int nsplit = Kp && dims.nsplit > 1 ? dims.nsplit : 1;
  OD_REQUIRE(nsplit <= 64, "od_prefix_attn: nsplit %d above 64", nsplit);
  const int64_t n_part = static_cast<int64_t>(dims.R) * dims.t * dims.Hq;
  if (nsplit > 1)
    OD_REQUIRE(workspace && aligned16(workspace) &&
                   workspace_bytes >= static_cast<int64_t>(sizeof(float)) * nsplit * n_part * (dims.D + 1),
               "od_prefix_attn: %d splits need a 16-byte aligned workspace of %lld bytes (od_prefix_attn_plan)", nsplit,
               (long long)(static_cast<int64_t>(sizeof(float)) * nsplit * n_part * (dims.D + 1)));
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_prefix_attn: no device error word");
  Params P;
  memset(&P, 0, sizeof(P));
  P.q = static_cast<const __nv_bfloat16*>(q);
  P.Kp = static_cast<const int8_t*>(Kp);
  P.Vp = static_cast<const int8_t*>(Vp);
  P.prefix_bf16 = pbf16 ? 1 : 0;
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
  P.R = dims.R;
  P.t = dims.t;
  P.T = dims.T;
  P.Lq = dims.Lq;
  P.Hq = dims.Hq;
  P.Hkv = dims.Hkv;
  P.rep = rep;
  P.tiles_per_group = static_cast<int>((gslots + NT * BM - 1) / (NT * BM));
  P.nsplit = nsplit;
  if (nsplit > 1) {
    P.part_o = static_cast<float*>(workspace);
    P.part_lse = P.part_o + static_cast<int64_t>(nsplit) * n_part * dims.D;
  }
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
    const int64_t tokens = static_cast<int64_t>(dims.R) * dims.t;
    if (!rc && BM % rep == 0 && tokens < (1LL << 31)) {
      rc = make_map_slots(&P.map_q, q, static_cast<uint64_t>(dims.D), static_cast<uint64_t>(dims.Hq),
                          static_cast<uint64_t>(tokens), rep);
      if (!rc) rc = make_map_slots(&P.map_o, o, static_cast<uint64_t>(dims.D), static_cast<uint64_t>(dims.Hq),
                                   static_cast<uint64_t>(tokens), rep);
      P.q_tma = 1;
    }
    if (!rc && Kp) {
      const uint64_t prows = static_cast<uint64_t>(dims.S) * dims.Hkv * dims.T;
      OD_REQUIRE(prows < (1ULL << 31), "od_prefix_attn: S * Hkv * T must be below 2^31");
      if (pbf16) {
        rc = make_map_bf16(&P.map_kp, Kp, static_cast<uint64_t>(dims.D), prows);
        if (!rc) rc = make_map_bf16(&P.map_vp, Vp, static_cast<uint64_t>(dims.D), prows);
      } else {
        rc = make_map_i8(&P.map_kp, Kp, static_cast<uint64_t>(dims.D), prows);
        if (!rc) rc = make_map_i8(&P.map_vp, Vp, static_cast<uint64_t>(dims.D), prows);
      }
    }
    if (rc) return rc;
  }
  const int64_t gx = G * P.tiles_per_group;
  OD_REQUIRE(gx < (1LL << 31) && dims.Hkv < 65536, "od_prefix_attn: grid too large");
  dim3 grid(static_cast<unsigned>(gx), dims.Hkv, nsplit);
  cudaStream_t st = as_stream(stream);
  const bool half_scale = Kp && !pbf16 && dims.scale_dtype == OD_F16;
  int rc = OD_OK;
#define OD_ATTN(NT_)                                                                                          \
  (dims.D == 128 ? (half_scale ? launch_attn<__half, 128, NT_>(P, grid, st)                                \
                               : launch_attn<__nv_bfloat16, 128, NT_>(P, grid, st))                        \
                 : (half_scale ? launch_attn<__half, 64, NT_>(P, grid, st)                                 \
                               : launch_attn<__nv_bfloat16, 64, NT_>(P, grid, st)))
  rc = NT == 1 ? OD_ATTN(1) : OD_ATTN(2);
#undef OD_ATTN
  if (rc != OD_OK || nsplit == 1) return rc;
  const unsigned mb = static_cast<unsigned>((n_part * 32 + 255) / 256);
  if (dims.D == 128)
    attn_merge_kernel<128><<<mb, 256, 0, st>>>(P.part_o, P.part_lse, nsplit, n_part, static_cast<int>(dims.t),
                                                dims.Hq, P.o, lse, P.err);
  else
    attn_merge_kernel<64><<<mb, 256, 0, st>>>(P.part_o, P.part_lse, nsplit, n_part, static_cast<int>(dims.t),
                                               dims.Hq, P.o, lse, P.err);
  OD_LAUNCH_CHECK();
  return ok();
}

extern "C" int od_prefix_attn_plan(const od_attn_dims* dims, int num_sms, int* nsplit, int64_t* workspace_bytes) {
  OD_REQUIRE(dims && nsplit && workspace_bytes, "od_prefix_attn_plan: null pointer");
  *nsplit = 1;
  *workspace_bytes = 0;
  if (dims->S <= 0 || dims->T <= 0 || dims->Hkv <= 0) return ok();
  const int64_t gslots = group_slots(*dims);
  const int64_t cta_slots = gslots <= BM ? BM : kMaxTiles * BM;
  const int64_t G = dims->max_group_rows > 1 ? dims->G : dims->R;
  const int64_t ctas = G * ((gslots + cta_slots - 1) / cta_slots) * dims->Hkv;
  const int n = plan_splits(ctas, (dims->T + BN - 1) / BN, num_sms);
  *nsplit = n;
  if (n > 1)
    *workspace_bytes = static_cast<int64_t>(sizeof(float)) * n * static_cast<int64_t>(dims->R) * dims->t * dims->Hq *
                       (dims->D + 1);
  return ok();
}

// ------------------------------------------------------------------------------------------------ no-alloc variant
// od_prefix_attn with the split workspace in a file-scope device array instead of a caller buffer. The array is
// part of the module's static device memory (one per device, mapped when the module loads); its address is taken
// once per device with cudaGetSymbolAddress. Nothing in it has to start at zero: every split writes the partial O
// and LSE of every slot it covers (a split left without keys writes O = 0, LSE = -inf) before the merge reads them.
// One array per device means calls on one device must be ordered (one stream, or synchronised streams): two
// in flight at once would share it.
namespace od {
namespace {
constexpr int64_t kNoAllocScratchBytes = 16LL << 20;
__device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

void* attn_scratch() {
  // Filled without a lock: threads that race on a device's first call all store the same address (the symbol's
  // address on that device), so a duplicate lookup is the only effect of the race.
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}
}  // namespace
}  // namespace od

extern "C" int od_prefix_attn_noalloc(const void* q, const void* Kp, const void* Vp, const void* ksc, const void* vsc,
                                      const int32_t* row_state, const int32_t* p_lo, const int32_t* p_hi,
                                      const uint8_t* pmask, const void* Kq, const void* Vq, const int32_t* row_q,
                                      const int32_t* q_len, const void* k_own, const void* v_own,
                                      const int32_t* own_lo, const int32_t* own_hi, const int32_t* row_groups,
                                      void* o, float* lse, od_attn_dims dims, void* stream) {
  const int nsplit = Kp && dims.nsplit > 1 ? dims.nsplit : 1;
  const int64_t need =
      nsplit > 1 ? static_cast<int64_t>(sizeof(float)) * nsplit * dims.R * dims.t * dims.Hq * (dims.D + 1) : 0;
  OD_REQUIRE(need <= kNoAllocScratchBytes,
             "od_prefix_attn_noalloc: %d splits need %lld bytes of scratch, the static scratch holds %lld (lower "
             "dims.nsplit or call od_prefix_attn with a workspace)",
             nsplit, (long long)need, (long long)kNoAllocScratchBytes);
  void* ws = nullptr;
  if (need > 0) {
    ws = attn_scratch();
    OD_REQUIRE(ws, "od_prefix_attn_noalloc: no address for the static scratch on this device");
  }
  return od_prefix_attn(q, Kp, Vp, ksc, vsc, row_state, p_lo, p_hi, pmask, Kq, Vq, row_q, q_len, k_own, v_own, own_lo,
                        own_hi, row_groups, o, lse, dims, ws, need, stream);
}

// ------------------------------------------------------------------------------------------------ failure detection
// Self-test of the bounded-wait path every kernel here relies on: one thread waits on an mbarrier nothing arrives
// on, with a caller-chosen cycle limit instead of the kernels' ~2 s, records kErrSelfTest in the device error word
// when the limit runs out and returns. The context stays usable (nothing faults, nothing keeps waiting).
namespace od {
namespace {
constexpr int32_t kErrSelfTest = 0x7F0001;

__global__ void bounded_wait_selftest_kernel(int64_t limit_cycles, int32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  const long long t0 = clock64();
  while (!mbar_try_wait(&bar, 0)) {
    if (clock64() - t0 > limit_cycles) {
      atomicCAS(err, 0, kErrSelfTest);
      return;
    }
  }
}
}  // namespace
}  // namespace od

extern "C" int od_selftest_bounded_wait(int64_t limit_cycles, void* stream) {
  OD_REQUIRE(limit_cycles > 0 && limit_cycles <= kWaitLimitCycles, "od_selftest_bounded_wait: limit out of range");
  int32_t* err = device_error_word();
  if (!err) return fail(OD_ECUDA, "od_selftest_bounded_wait: no device error word");
  bounded_wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(limit_cycles, err);
  OD_LAUNCH_CHECK();
  return ok();
}
