// Decode GEMV (M <= 16) on the integer tensor-core path: u8 codes x 8-bit activation digits.
//
// Replaces, like the other decode GEMVs, the reference's per-call dequant + F.linear for small M
// (packed_gptq_linear.py:66-74, fused_int4_linear.py:127-272 at decode sizes).
//
// Why: the 16-bit decode GEMV (gemv_tma.cuh) spends most of its issue slots turning nibbles into
// bf16 pairs (3 shifts + 4 lop3 per 32-bit word: bf16's 7-bit mantissa holds one nibble position),
// on an extra MMA against ones for the activation sums, and on the per-group float fix-up. Here:
//   * x8_prepare_kernel (one launch per call; it also does the act-order gather that the 16-bit
//     path launches separately) writes each token's activations per 128-k stage as exact 16-bit
//     fixed point X = RNE(x * 2^-e), e = floor(log2 max|x|) - 14 over the stage, split into two
//     8-bit digits X = 256 d1 + d0 (d0 unsigned, d1 signed), with the stage's 2^e and the sums of
//     X over each 32-k quarter of the stage. A bf16 (fp16) value whose exponent is within 7 (5)
//     of the stage maximum's is represented exactly; smaller values are rounded to 2^e, an error
//     of at most 2^-16 of the stage's largest |x| per value.
//   * the GEMV unpacks a 32-bit word of 8 codes into two registers of 4 bytes with one shift and
//     two masks (even and odd nibble positions) and runs mma.sync.m16n8k32 u8 x u8 (low digit) and
//     u8 x s8 (high digit) into int32 accumulators; per segment (a group, or a stage when the group
//     is longer) D = C0 + 256 C1 - z * sum(X) is exact in int32 and acc += s * 2^e * float(D).
//   So the per-weight work is 3 integer operations per 8 codes plus 1 MMA per 16 codes and token
//   tile, and the zero-point correction is integer arithmetic.
//
// Fragment layout (m16n8k32, 8-bit A row-major, B column-major): lane (g = lane / 4, t = lane % 4)
// holds the 128-bit vector qweight[4j + t][n0 + 4g .. 4g + 3] of step j (4 columns x 8 k), as in the
// 16-bit kernel. A register a0 = even nibbles (k 0, 2, 4, 6 of its word) of column 4g + 2beta (MMA
// row g), a1 = the same for column 4g + 2beta + 1 (row g + 8), a2 / a3 = odd nibbles. The MMA's k
// slots 4t..4t+3 / 16+4t..16+4t+3 are therefore the even / odd positions of word row 4j + t, and the
// prepared activations store each word's digits in that order: [d0 even | d0 odd | d1 even | d1 odd].
//
// Pipeline, split-K, failure handling and programmatic dependent launch follow gemv_tma.cuh: one TMA
// producer warp fills an mbarrier ring with the 128-k stage of a 128-column tile (four 32-column
// weight slabs with the 128-byte swizzle, the stage's scale and zero rows, the prepared activation
// rows of 8 MT tokens); 8 consumer warps (4 column warps x 2 stage halves) read shared memory only.
//
// Split-K reduction. With two splits per column tile (the wide layers) the splits are one
// thread-block cluster (launched with cluster dims (1, 2, 1)): each CTA leaves its partial sums in
// its own shared memory and arrives on an mbarrier of the leader (split 0); the leader reads the
// partials over distributed shared memory in split order (deterministic), applies the epilogue and
// writes the tile, then releases the other CTA, which waits so that its shared memory outlives the
// leader's reads. That replaces the global-memory reduction (partials to a workspace, a fence, an
// atomic ticket and a re-read by the last CTA), a chain of dependent L2 round trips at the end of
// the layer. Larger clusters measured slower (their CTAs must be co-scheduled on one GPC, which
// delays launches while the previous layer's CTAs still hold SMs), so layers split more ways keep
// the global reduction. Every wait is bounded.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace oc {

constexpr int kX8StageK = 128;                 // k per stage (16 words of 8 codes)
constexpr int kX8RowBytes = 320;               // per (token, stage): 16 words x 16 B of digits + 64 B record
constexpr int kX8RowWords = kX8RowBytes / 4;   // 80 (TMA box inner extent, in 32-bit elements)
constexpr int kX8RecOff = 256;                 // record: int32 sum X per 32-k quarter [4], then float 2^e
// The record is padded to 64 B so consecutive token rows start 4 16-byte chunks apart in shared
// memory: the two token rows that one quarter-warp reads then use disjoint banks.

// ---- activation preparation ------------------------------------------------------------------
// One thread per (token, 8-k word of the kernel's K order); the 16 threads of a half-warp (all
// active: half_mask) are one stage and write its 320-byte row `row`. x element k of the kernel
// order is x[m, kperm[k]] (kperm null: x[m, k]); indices outside [0, K) and words past Kp give 0.
// The permutation is part of the layer, so it is read before waiting for the kernel that wrote x.
template <bool BF16>
__device__ __forceinline__ void x8_prepare_word(const uint16_t* __restrict__ x, long long ldx, int K,
                                                const int32_t* __restrict__ kperm, int Kp, int m, int kb, int w,
                                                unsigned half_mask, uint8_t* __restrict__ row) {
  const int k0 = kb * kX8StageK + 8 * w;  // first k (kernel order) of this word
  const bool in = k0 < Kp;                // Kp is a multiple of 8: a word is wholly in or out
  int src[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int s = -1;
    if (in) s = kperm ? __ldg(kperm + k0 + i) : k0 + i;
    src[i] = (s >= 0 && s < K) ? s : -1;
  }
  griddep_wait();
  const uint16_t* xr = x + (long long)m * ldx;
  float v[8];
  if (!kperm && in && k0 + 8 <= K) {
    const uint4 q = *reinterpret_cast<const uint4*>(xr + k0);
    const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bits_to_f32((uint16_t)(qq[i] & 0xFFFFu), BF16 ? kBF16 : kF16);
      v[2 * i + 1] = bits_to_f32((uint16_t)(qq[i] >> 16), BF16 ? kBF16 : kF16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = src[i] >= 0 ? bits_to_f32(xr[src[i]], BF16 ? kBF16 : kF16) : 0.f;
  }

  // stage maximum (non-finite values make it NaN or inf)
  float amax = 0.f;
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    bad |= !(a <= 3.4028235e38f);  // NaN or inf
    amax = fmaxf(amax, a);
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    amax = fmaxf(amax, __shfl_xor_sync(half_mask, amax, o));
    bad |= __shfl_xor_sync(half_mask, (int)bad, o) != 0;
  }

  int X[8];
  float scale;
  if (bad) {
#pragma unroll
    for (int i = 0; i < 8; ++i) X[i] = 0;
    scale = __uint_as_float(0x7FC00000u);  // NaN: every output of this token becomes NaN
  } else if (amax == 0.f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) X[i] = 0;
    scale = 0.f;
  } else {
    // E = floor(log2(amax)) from the exponent field (subnormal maxima lifted by 2^64 first)
    float a = amax;
    int adj = 0;
    if (a < 1.17549435e-38f) {
      a *= 18446744073709551616.f;  // 2^64, exact
      adj = 64;
    }
    const int E = (int)((__float_as_uint(a) >> 23) & 0xFFu) - 127 - adj;
    // X = RNE(v * 2^(14 - E)); the factor is applied as two powers of two that are each
    // representable, so the scaling is exact and amax maps to [2^14, 2^15)
    const int sh = 14 - E;                       // in [-113, 163]
    const int sh1 = sh > 120 ? 120 : sh;
    const int sh2 = sh - sh1;                    // 0 unless sh > 120
    const float f1 = __uint_as_float((uint32_t)(sh1 + 127) << 23);
    const float f2 = __uint_as_float((uint32_t)(sh2 + 127) << 23);
#pragma unroll
    for (int i = 0; i < 8; ++i) X[i] = __float2int_rn((v[i] * f1) * f2);
    // 2^(E - 14) as a float; below the subnormal range the stage's contribution is dropped
    const int es = E - 14;
    scale = es >= -126 ? __uint_as_float((uint32_t)(es + 127) << 23)
                       : (es >= -149 ? __uint_as_float(1u << (es + 149)) : 0.f);
  }

  // sum of X over the 4 words (32 k) of this lane's quarter
  int sx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) sx += X[i];
  sx += __shfl_xor_sync(half_mask, sx, 1);
  sx += __shfl_xor_sync(half_mask, sx, 2);

  // digits in MMA order: [d0 even | d0 odd | d1 even | d1 odd], even = k 0, 2, 4, 6 of the word
  uint32_t d0e = 0, d0o = 0, d1e = 0, d1o = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo_e = (uint32_t)X[2 * i] & 0xFFu, lo_o = (uint32_t)X[2 * i + 1] & 0xFFu;
    const uint32_t hi_e = (uint32_t)(X[2 * i] >> 8) & 0xFFu, hi_o = (uint32_t)(X[2 * i + 1] >> 8) & 0xFFu;
    d0e |= lo_e << (8 * i);
    d0o |= lo_o << (8 * i);
    d1e |= hi_e << (8 * i);
    d1o |= hi_o << (8 * i);
  }
  *reinterpret_cast<uint4*>(row + 16 * w) = make_uint4(d0e, d0o, d1e, d1o);
  if ((w & 3) == 0) *reinterpret_cast<int*>(row + kX8RecOff + (w >> 2) * 4) = sx;
  if (w == 0) *reinterpret_cast<float*>(row + kX8RecOff + 16) = scale;
}

// The preparation as its own launch, into the workspace layout [M][stages][320 B].
template <bool BF16>
__global__ void __launch_bounds__(256) x8_prepare_kernel(const uint16_t* __restrict__ x, long long ldx, int M, int K,
                                                         const int32_t* __restrict__ kperm, int Kp, int KB,
                                                         uint8_t* __restrict__ out) {
  griddep_launch_dependents();
  const long long total = (long long)M * KB * 16;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // total is a multiple of 16, so a half-warp is either wholly inside or wholly past it
  if (gid >= total) return;
  const unsigned half_mask = 0xFFFFu << (threadIdx.x & 16);
  const int m = (int)(gid / ((long long)KB * 16));
  const int rem = (int)(gid - (long long)m * KB * 16);
  const int kb = rem >> 4, w = rem & 15;
  x8_prepare_word<BF16>(x, ldx, K, kperm, Kp, m, kb, w, half_mask, out + ((long long)m * KB + kb) * kX8RowBytes);
}

// ---- the GEMV ----------------------------------------------------------------------------------
// Shared-memory stage of XR activation rows and SPS scale / zero rows; the ring is as deep as
// about 98 KB allows (two CTAs per SM), so a 2-row box (M <= 2) buys three more weight stages in
// flight than an 8-row one.
// Every slot is a multiple of 128 bytes: a tiled TMA copy needs a 128-byte aligned shared-memory
// destination (1024 bytes for the 128-byte swizzle of the weight slabs).
// PREP (the host uses it for one token without a K permutation; the kernel takes M <= 2): the CTA
// prepares the activations of its whole K split itself, into a region of kPrepMaxStages x
// [2 tokens][320 B] after the ring, instead of a separate launch writing them to the workspace and
// a TMA copy per stage bringing them back (the ring then carries no activation slot; kSmemBytes
// leaves out the prepared region, which the launch adds).
constexpr int kPrepMaxStages = 20;
template <int MT, int SPS, int XR, bool PREP = false>
struct G8Cfg {
  static constexpr int kWBytes = 4 * 16 * 128;           // four [16 rows][32 words] slabs, 128B-swizzled
  static constexpr int kSBytes = SPS * kGemvCols * 2;    // one scale row per segment
  static constexpr int kZBytes = (SPS * (kGemvCols / 8) * 4 + 127) / 128 * 128;  // zero rows, padded
  static constexpr int kXBytes = PREP ? 0 : XR * kX8RowBytes;  // [XR tokens][320 B]
  static constexpr int kStage = kWBytes + kSBytes + kZBytes + kXBytes;
  static constexpr int kBudget = (PREP ? 86 : (MT == 1 ? 98 : 94)) * 1024;
  static constexpr int kDepth = kBudget / kStage > 12 ? 12 : kBudget / kStage;
  static constexpr int kWOff = 0;
  static constexpr int kSOff = kDepth * kWBytes;
  static constexpr int kZOff = kSOff + kDepth * kSBytes;
  static constexpr int kXOff = kZOff + kDepth * kZBytes;
  static constexpr int kBarOff = kXOff + kDepth * kXBytes;
  static constexpr int kPrepOff = (kBarOff + 2 * kDepth * 8 + 16 + 127) / 128 * 128;
  static constexpr int kPrepRowBytes = 2 * kX8RowBytes;  // one stage: [2 tokens][320 B]
  static constexpr int kSmemBytes = (PREP ? kPrepOff : kBarOff + 2 * kDepth * 8 + 16) + 1024 /*align*/;
  static_assert(!PREP || (MT == 1 && XR == 2), "the CTA prepares activations for up to 2 tokens");
  static_assert(kWBytes % 1024 == 0 && kSBytes % 128 == 0 && kZBytes % 128 == 0 && kXBytes % 128 == 0,
                "TMA destinations: 1024-byte swizzled weight slabs, 128-byte aligned other slots");
  static_assert(kSOff % 128 == 0 && kZOff % 128 == 0 && kXOff % 128 == 0, "128-byte aligned slot arrays");
};

// D (+)= A * B, u8 A; B u8 (S8B false) or s8; ZERO: the accumulator starts at 0
template <bool S8B, bool ZERO>
__device__ __forceinline__ void mma_i8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (ZERO) {
    if constexpr (S8B)
      asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%10,%10,%10,%10};"
          : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
          : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
    else
      asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%10,%10,%10,%10};"
          : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
          : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
  } else {
    if constexpr (S8B)
      asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%0,%1,%2,%3};"
          : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
          : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
      asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%0,%1,%2,%3};"
          : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
          : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// SPS: segments per stage (4: groups of 32 rows, 2: groups of 64, 1: groups of 128 * n, flushed
// once per stage). ODD: tokens 2t + 1 exist (M > 1); with M == 1 the fix-up skips them. XR: rows of
// the activation box (2 for M <= 2, else 8 MT; rows past M are zero-filled by the copy).
// gp.cluster: the splits of a tile reduce in their cluster (launched with cluster dims
// (1, splits, 1)); otherwise through the workspace, as the other decode GEMVs.
// PREP: the consumers prepare the split's activations from gp.x8 / gp.kperm (x8_prepare_word) before
// their first stage; tmap_x is unused.
template <bool BF16, int MT, int SPS, bool ODD, int XR, bool PREP = false>
__global__ void __launch_bounds__(kGtThreads, 2)
    gptq_gemv_i8_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                        const __grid_constant__ CUtensorMap tmap_z, const __grid_constant__ CUtensorMap tmap_x,
                        const GtParams gp) {
  using Cfg = G8Cfg<MT, SPS, XR, PREP>;
  constexpr int kCons = kGtConsumerWarps;
  const GemvParams& p = gp.g;
  extern __shared__ __align__(1024) uint8_t g8_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(g8_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* empty = full + Cfg::kDepth;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + Cfg::kDepth);
  __shared__ __align__(16) float red[kGemvWarpsN][32][MT * 8];
  __shared__ __align__(8) uint64_t cl_bar[2];  // [0] the leader's: partials ready; [1] the others': released
  __shared__ int cta_failed;
  __shared__ int is_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;  // split == rank in the (1, splits, 1) cluster
  const int nsplit = gridDim.y;
  const int KB = (p.Kp + kX8StageK - 1) / kX8StageK;
  const int kb0 = split * gp.kb_per_split;
  const int kb1 = min(KB, kb0 + gp.kb_per_split);
  const int nst = kb1 - kb0;
  const int col0 = tile * kGemvCols;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kDepth; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the 4 column warps that consume a stage
    }
    mbar_init(&cl_bar[0], nsplit);
    mbar_init(&cl_bar[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // every CTA of the cluster has initialised its barriers once this phase completes; the consumers
  // wait for it before their first access to another CTA's shared memory
  if (gp.cluster) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  griddep_launch_dependents();

  if (warp == kCons) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_s);
      tma_prefetch_desc(&tmap_z);
      if constexpr (!PREP) tma_prefetch_desc(&tmap_x);
      // bytes the copies of one stage deliver (the zero slot's padding is not copied)
      const uint32_t bytes = Cfg::kWBytes + SPS * (kGemvCols * 2 + kGemvCols / 2) + Cfg::kXBytes;
      int armed[Cfg::kDepth];
      for (int i = 0; i < Cfg::kDepth; ++i) armed[i] = -1;
      auto load_wsz = [&](int i) {
        const int s = i % Cfg::kDepth;
        const int kb = kb0 + i;
        mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(smem + Cfg::kWOff + s * Cfg::kWBytes + c * 2048, &tmap_w, &full[s], col0 + 32 * c, kb * 16);
        const int g0 = (kb * kX8StageK) / p.gs;
        tma_load_2d(smem + Cfg::kSOff + s * Cfg::kSBytes, &tmap_s, &full[s], col0, g0);
        tma_load_2d(smem + Cfg::kZOff + s * Cfg::kZBytes, &tmap_z, &full[s], col0 / 8, g0);
        armed[s] = (i / Cfg::kDepth) & 1;
      };
      auto load_x = [&](int i) {
        const int s = i % Cfg::kDepth;
        tma_load_2d(smem + Cfg::kXOff + s * Cfg::kXBytes, &tmap_x, &full[s], (kb0 + i) * kX8RowWords, 0);
      };
      const int stall = (blockIdx.x == 0 && blockIdx.y == 0) ? gp.stall_stage - 1 : -1;
      // weights of the first stages before the previous kernel (the activation preparation) ends;
      // with PREP the producer copies layer constants only and never waits for it
      const int pre = nst < Cfg::kDepth ? nst : Cfg::kDepth;
      for (int i = 0; i < pre; ++i)
        if (i != stall) load_wsz(i);
      if constexpr (!PREP) {
        griddep_wait();
        for (int i = 0; i < pre; ++i)
          if (i != stall) load_x(i);
      }
      for (int i = pre; i < nst; ++i) {
        const int s = i % Cfg::kDepth;
        if (!mbar_wait_ns(&empty[s], ((i / Cfg::kDepth) & 1) ^ 1, abort_flag, kDevErrWEmpty, gp.wait_ns)) break;
        if (i == stall) continue;
        load_wsz(i);
        if constexpr (!PREP) load_x(i);
      }
      // the CTA must not exit with a bulk copy in flight: wait (bounded) for every armed stage
      for (int s = 0; s < Cfg::kDepth; ++s)
        if (armed[s] >= 0) mbar_drain(&full[s], armed[s]);
    }
    return;  // no further __syncthreads below
  }

  // -------------------------------------------------------------------- consumers
  const int wn = warp & 3, kh = warp >> 2;
  const int g = lane >> 2, t = lane & 3;
  const int cw = wn * 32 + 4 * g;  // column within the tile
  const int col = col0 + cw;
  const int zsh = 4 * (col & 7);
  constexpr int kQuartersPerSeg = 4 / SPS;

  float acc[MT][2][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;
  int c0[MT][2][4], c1[MT][2][4];
  float sj[4];
  int zj[4];

  auto load_sz = [&](const uint8_t* srow, const uint8_t* zrow) {
    const uint2 sv = *reinterpret_cast<const uint2*>(srow + cw * 2);
    uint32_t zw = *reinterpret_cast<const uint32_t*>(zrow + (cw / 8) * 4);
    if (p.v1) zw = ((zw & 0x77777777u) + 0x11111111u) ^ (zw & 0x88888888u);  // (z + 1) mod 16 per field
    if (p.s_dtype == kF16) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
      sj[0] = a.x; sj[1] = a.y; sj[2] = b.x; sj[3] = b.y;
    } else {
      sj[0] = __uint_as_float(sv.x << 16);
      sj[1] = __uint_as_float(sv.x & 0xFFFF0000u);
      sj[2] = __uint_as_float(sv.y << 16);
      sj[3] = __uint_as_float(sv.y & 0xFFFF0000u);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) zj[j] = (int)((zw >> (zsh + 4 * j)) & 0xFu);
  };
  // acc += s * 2^e * (C0 + 256 C1 - z * sum X) over the segment of quarters [q0, q0 + kQuartersPerSeg)
  auto flush = [&](const uint8_t* xst, int q0) {
#pragma unroll
    for (int a = 0; a < MT; ++a) {
#pragma unroll
      for (int h = 0; h < (ODD ? 2 : 1); ++h) {
        const int tok = 8 * a + 2 * t + h;
        const uint8_t* rec = xst + (tok < XR ? tok : 0) * kX8RowBytes + kX8RecOff;
        int sx;
        if constexpr (kQuartersPerSeg == 4) {
          const int4 q = *reinterpret_cast<const int4*>(rec);
          sx = (q.x + q.y) + (q.z + q.w);
        } else if constexpr (kQuartersPerSeg == 2) {
          const int2 q = *reinterpret_cast<const int2*>(rec + 4 * q0);
          sx = q.x + q.y;
        } else {
          sx = *reinterpret_cast<const int*>(rec + 4 * q0);
        }
        float sc = *reinterpret_cast<const float*>(rec + 16);
        if (tok >= XR) {  // a token row outside the box (never stored)
          sx = 0;
          sc = 0.f;
        }
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int c = 2 * cc + h;   // c & 1 = token parity, c >> 1 = second column of the pair
            const int j = 2 * b + cc;   // column within the lane's four
            const int d = c0[a][b][c] + 256 * c1[a][b][c] - zj[j] * sx;
            acc[a][b][c] = fmaf(sj[j] * sc, (float)d, acc[a][b][c]);
          }
      }
    }
  };

  if constexpr (PREP) {
    // this split's activations, [stage][token][320 B], one half-warp per (token, stage); the weight
    // stages keep landing meanwhile
    const int items = p.M * nst * 16;   // a multiple of 16: half-warps are wholly in or out
    const unsigned half_mask = 0xFFFFu << (threadIdx.x & 16);
    for (int base = 0; base < items; base += kCons * 32) {
      const int it = base + threadIdx.x;
      if (it < items) {
        const int m = it / (nst * 16);
        const int rem = it - m * nst * 16;
        const int j = rem >> 4;
        x8_prepare_word<BF16>(p.x, p.ldx, gp.k_in, gp.kperm, p.Kp, m, kb0 + j, rem & 15, half_mask,
                              smem + Cfg::kPrepOff + j * Cfg::kPrepRowBytes + m * kX8RowBytes);
      }
    }
    named_bar_sync(4, kCons * 32);
  }

  bool ok = true;
  for (int i = kh; i < nst; i += 2) {
    const int s = i % Cfg::kDepth;
    if (!mbar_wait_ns(&full[s], (i / Cfg::kDepth) & 1, abort_flag, kDevErrWFull, gp.wait_ns)) {
      ok = false;
      break;
    }
    const uint8_t* wst = smem + Cfg::kWOff + s * Cfg::kWBytes + wn * 2048;
    const uint8_t* sst = smem + Cfg::kSOff + s * Cfg::kSBytes;
    const uint8_t* zst = smem + Cfg::kZOff + s * Cfg::kZBytes;
    const uint8_t* xst = PREP ? smem + Cfg::kPrepOff + i * Cfg::kPrepRowBytes : smem + Cfg::kXOff + s * Cfg::kXBytes;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 32-k step within the stage
      constexpr int kStepsPerSeg = 4 / SPS;
      const bool seg_first = (j % kStepsPerSeg) == 0;
      if (seg_first) {
        const int srow = j / kStepsPerSeg;
        load_sz(sst + srow * (kGemvCols * 2), zst + srow * (kGemvCols / 2));
      }
      const int r = 4 * j + t;  // word row within the slab
      const uint4 w = *reinterpret_cast<const uint4*>(wst + r * 128 + ((g ^ (r & 7)) << 4));
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
      uint32_t ev[4], od[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        ev[q] = wv[q] & 0x0F0F0F0Fu;
        od[q] = (wv[q] >> 4) & 0x0F0F0F0Fu;
      }
#pragma unroll
      for (int a = 0; a < MT; ++a) {
        const int tok = g + 8 * a;
        const uint4 xd = (tok < p.M && tok < XR) ? *reinterpret_cast<const uint4*>(xst + tok * kX8RowBytes + 16 * r)
                                                 : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const uint32_t af[4] = {ev[2 * b], ev[2 * b + 1], od[2 * b], od[2 * b + 1]};
          if (seg_first) {
            mma_i8<false, true>(c0[a][b], af, xd.x, xd.y);
            mma_i8<true, true>(c1[a][b], af, xd.z, xd.w);
          } else {
            mma_i8<false, false>(c0[a][b], af, xd.x, xd.y);
            mma_i8<true, false>(c1[a][b], af, xd.z, xd.w);
          }
        }
      }
      if ((j % kStepsPerSeg) == kStepsPerSeg - 1) flush(xst, (j / kStepsPerSeg) * kQuartersPerSeg);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // reduce the two stage halves of the CTA (named barrier over the consumer warps)
  if (kh == 1) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[wn][lane][a * 8 + b * 4 + c] = acc[a][b][c];
  }
  const bool any_fail = named_bar_or(1, kCons * 32, !ok);
  if (kh == 0) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[a][b][c] += red[wn][lane][a * 8 + b * 4 + c];
          red[wn][lane][a * 8 + b * 4 + c] = acc[a][b][c];  // this CTA's partial, read by the leader
        }
  }
  if (!gp.cluster) {
    griddep_wait();  // the previous kernel is done with the workspace and the output
    // a failed CTA (its error is recorded) still takes its split-K ticket and writes nothing
    gemv_finish_n<BF16, MT>(p, acc, kh, col, t, tile, split, &is_last, kCons * 32, any_fail);
    return;
  }
  if (threadIdx.x == 0) cta_failed = any_fail ? 1 : 0;
  named_bar_sync(2, kCons * 32);
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
    mbar_arrive_cluster(mapa_shared(&cl_bar[0], 0));
  }
  if (split != 0) {
    // keep this CTA's shared memory alive until the leader has read it
    if (threadIdx.x == 0) mbar_wait_cluster_ns(&cl_bar[1], 0, kDevErrCluster, OC_WAIT_NS);
    return;
  }
  if (kh == 1) return;
  // ---- leader: the tile's partials in split order
  const int nthr = 128;  // the 4 kh == 0 warps
  bool fail = !mbar_wait_cluster_ns(&cl_bar[0], 0, kDevErrCluster, OC_WAIT_NS);
  float sum[MT * 8];
#pragma unroll
  for (int i = 0; i < MT * 8; ++i) sum[i] = 0.f;
  for (int sp = 0; sp < nsplit && !fail; ++sp) {
    fail |= ld_dsmem_s32(mapa_shared(&cta_failed, sp)) != 0;
    const uint32_t base = mapa_shared(&red[wn][lane][0], sp);
#pragma unroll
    for (int i = 0; i < MT * 2; ++i) {
      const float4 v = ld_dsmem_f4(base + 16 * i);
      sum[4 * i] += v.x;
      sum[4 * i + 1] += v.y;
      sum[4 * i + 2] += v.z;
      sum[4 * i + 3] += v.w;
    }
  }
  // the sums consumed every value read, so the other CTAs can go once all leader threads are here
  fail = named_bar_or(3, nthr, fail);
  if (threadIdx.x == 0)
    for (int sp = 1; sp < nsplit; ++sp) mbar_arrive_cluster(mapa_shared(&cl_bar[1], sp));
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = sum[a * 8 + b * 4 + c];
  griddep_wait();  // the previous kernel is done with the output
  GemvParams q = p;
  q.splits = 1;  // the sum over splits is complete: epilogue and store only
  gemv_finish_n<BF16, MT>(q, acc, 0, col, t, tile, 0, &is_last, nthr, fail);
}

}  // namespace oc
