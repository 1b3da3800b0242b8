// Decode-sized (M <= 16) factored GEMV fed by TMA, for uniform groups of 32, 64 or a multiple
// of 128 rows (every GPTQ layout of configs 0-2). Same arithmetic as gptq_gemv_fact_kernel
// (gemv.cuh): the tensor cores multiply raw magic-biased codes (M + q) by the activations and
// each group's scale / zero is applied once to the fp32 sums.
//
// Why a separate kernel: with per-lane cp.async the decode GEMV is issue-bound (address and
// ring bookkeeping per 16-byte vector). Here one producer lane moves a whole 128-k block of a
// 128-column tile per stage with five TMA copies (four 32-column weight slabs with the 128-byte
// swizzle, the block's scale and zero rows, the activation rows), and the eight consumer warps
// only read shared memory, extract nibbles and issue MMAs.
//
// Launch overlap: the kernel is launched with programmatic stream serialization. Every CTA lets
// the next kernel in the stream launch at once (griddepcontrol.launch_dependents), and the
// producer streams the first stages of weights, which no earlier kernel writes, before it waits
// for the previous kernel (griddepcontrol.wait); activations and every global write (split-K
// partials, tickets, output) come after that wait.
//
// 8-bit layers (WB = 8): a 32-bit word holds 4 k of one column, so a stage of 16 word rows
// covers 64 k. bf16 cannot hold M + q exactly for q >= 128, so each byte is split into its two
// nibbles, both multiplied as magic-biased 4-bit codes into separate fp32 accumulators, and the
// group flush combines them: s * (C_lo + 16 C_hi) - s * (17 M + z) * sum(x) = s * sum(x (q - z)).
// The MMA count per weight byte is the 4-bit kernel's.
//
// CTA: 8 consumer warps (4 column warps x 2 stage halves; warp (wn, kh) takes every other
// stage, kh, kh + 2, ..., all 4 steps of it, so a group of 128 rows is flushed once per 4
// steps) + 1 producer warp. Split-K over CTAs as in gemv.cuh (deterministic
// last-CTA reduction). Every mbarrier wait is bounded; on timeout the kernel records an error
// code, drains its own copies and skips its writes.
#pragma once

#include "common.cuh"
#include "gemv.cuh"

namespace oc {

constexpr int kGtConsumerWarps = 8;
constexpr int kGtThreads = 32 * (kGtConsumerWarps + 1);
constexpr int kGtBK = 128;  // 4-bit k per stage: 16 word rows, 4 MMA steps of 32 k (8-bit: 64 k)

// k covered by one stage of 16 word rows
template <int WB>
constexpr int gt_stage_k() { return WB == 8 ? 64 : kGtBK; }

template <int MT>
struct GtCfg {
  static constexpr int kDepth = MT == 1 ? 8 : 6;
  static constexpr int kWBytes = 4 * 16 * 128;          // four [16 rows][32 words] slabs, 128B-swizzled
  static constexpr int kSBytes = 4 * kGemvCols * 2;     // up to 4 scale rows (groups of 32)
  static constexpr int kZBytes = 4 * (kGemvCols / 8) * 4;  // 4 rows of 4-bit zeros = 2 rows of 8-bit
  static constexpr int kXBytes = 8 * MT * kGtBK * 2;    // [8 MT tokens][128 k]
  static constexpr int kWOff = 0;
  static constexpr int kSOff = kDepth * kWBytes;
  static constexpr int kZOff = kSOff + kDepth * kSBytes;
  static constexpr int kXOff = kZOff + kDepth * kZBytes;
  static constexpr int kBarOff = kXOff + kDepth * kXBytes;
  static constexpr int kSmemBytes = kBarOff + 2 * kDepth * 8 + 16 + 1024 /*align*/;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

struct GtParams {
  GemvParams g;
  int rows_sz;        // scale/zero rows per stage: stage k / gs when gs divides it, else 1
  int kb_per_split;   // stages per split
  unsigned long long wait_ns;  // bound of the pipeline waits (drains keep OC_WAIT_NS)
  int stall_stage;    // failure test only: > 0 leaves stage stall_stage - 1 of CTA (0, 0) unissued,
                      // so its consumers' wait runs out; 0 in normal use
  int cluster;        // integer GEMV: the K splits of a tile are one cluster and reduce in it
  const int32_t* kperm;  // integer GEMV preparing its own activations (g.x in the caller's K
  int k_in;              // order, g.ldx): the layer's K permutation (or null) and its K
};

template <bool BF16, int MT, int WB = 4>
__global__ void __launch_bounds__(kGtThreads, 2)
    gptq_gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                         const __grid_constant__ CUtensorMap tmap_z, const __grid_constant__ CUtensorMap tmap_x,
                         const GtParams gp) {
  using P = Pair<BF16>;
  using Cfg = GtCfg<MT>;
  const GemvParams& p = gp.g;
  extern __shared__ __align__(1024) uint8_t gt_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gt_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* empty = full + Cfg::kDepth;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + Cfg::kDepth);
  __shared__ float red[kGemvWarpsN][32][MT * 8];
  __shared__ int is_last;

  static_assert(WB == 4 || WB == 8, "4- or 8-bit codes");
  constexpr int KS = gt_stage_k<WB>();   // k per stage
  constexpr int KSTEP = KS / 4;          // k per MMA step (4 word rows)
  constexpr int kZRowBytes = kGemvCols * WB / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int KB = (p.Kp + KS - 1) / KS;
  const int kb0 = split * gp.kb_per_split;
  const int kb1 = min(KB, kb0 + gp.kb_per_split);
  const int nst = kb1 - kb0;
  const int col0 = tile * kGemvCols;

  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::kDepth; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGtConsumerWarps / 2);  // the 4 column warps of one stage half
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kGtConsumerWarps) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_s);
      tma_prefetch_desc(&tmap_z);
      tma_prefetch_desc(&tmap_x);
      const uint32_t bytes = Cfg::kWBytes + gp.rows_sz * (kGemvCols * 2 + kZRowBytes) + 8 * MT * KS * 2;
      int armed[Cfg::kDepth];
      for (int i = 0; i < Cfg::kDepth; ++i) armed[i] = -1;
      auto load_wsz = [&](int i) {
        const int s = i % Cfg::kDepth;
        const int kb = kb0 + i;
        mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(smem + Cfg::kWOff + s * Cfg::kWBytes + c * 2048, &tmap_w, &full[s], col0 + 32 * c, kb * 16);
        const int g0 = (kb * KS) / p.gs;
        tma_load_2d(smem + Cfg::kSOff + s * Cfg::kSBytes, &tmap_s, &full[s], col0, g0);
        tma_load_2d(smem + Cfg::kZOff + s * Cfg::kZBytes, &tmap_z, &full[s], col0 * WB / 32, g0);
        armed[s] = (i / Cfg::kDepth) & 1;
      };
      auto load_x = [&](int i) {
        const int s = i % Cfg::kDepth;
        tma_load_2d(smem + Cfg::kXOff + s * Cfg::kXBytes, &tmap_x, &full[s], (kb0 + i) * KS, 0);
      };
      const int stall = (blockIdx.x == 0 && blockIdx.y == 0) ? gp.stall_stage - 1 : -1;
      // weights of the first stages before the previous kernel has finished
      const int pre = nst < Cfg::kDepth ? nst : Cfg::kDepth;
      for (int i = 0; i < pre; ++i)
        if (i != stall) load_wsz(i);
      griddep_wait();
      for (int i = 0; i < pre; ++i)
        if (i != stall) load_x(i);
      for (int i = pre; i < nst; ++i) {
        const int s = i % Cfg::kDepth;
        if (!mbar_wait_ns(&empty[s], ((i / Cfg::kDepth) & 1) ^ 1, abort_flag, kDevErrWEmpty, gp.wait_ns)) break;
        if (i == stall) continue;
        load_wsz(i);
        load_x(i);
      }
      // Wait (bounded) for every copy this lane issued to land, whatever happened to the
      // consumers: the CTA must not exit with a bulk copy in flight. Copies already consumed
      // have completed their phase, so those waits return at once.
      for (int s = 0; s < Cfg::kDepth; ++s)
        if (armed[s] >= 0) mbar_drain(&full[s], armed[s]);
    }
    return;  // the producer warp takes no part in the reduction below (no further __syncthreads)
  }

  // -------------------------------------------------------------------- consumers
  const int wn = warp & 3, kh = warp >> 2;
  const int g = lane >> 2, t = lane & 3;
  const int cw = wn * 32 + 4 * g;  // column within the tile
  const int col = col0 + cw;
  const int zsh = WB == 8 ? 0 : 4 * (col & 7);
  // steps per group when a stage holds several groups: 1 or 2 (groups of 32 or 64 rows), so the
  // per-step tests below are a mask and a shift
  const int spg_step = p.gs / KSTEP;
  const int spg_shift = spg_step >= 2 ? 1 : 0;
  const uint32_t ones = BF16 ? 0x3F803F80u : 0x3C003C00u;
  const uint32_t ones4[4] = {ones, ones, ones, ones};

  // cg: codes (low nibbles for 8-bit) x activations; ch: high nibbles (8-bit only)
  constexpr int NH = WB == 8 ? MT : 1;
  float acc[MT][2][4], cg[MT][2][4], ch[NH][2][4], xo[MT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a) {
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = cg[a][b][c] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) xo[a][c] = 0.f;
  }
#pragma unroll
  for (int a = 0; a < NH; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) ch[a][b][c] = 0.f;
  float sj[4] = {0.f, 0.f, 0.f, 0.f}, czj[4] = {0.f, 0.f, 0.f, 0.f};
  auto flush = [&]() {
#pragma unroll
    for (int a = 0; a < MT; ++a) {
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = 2 * b + (c >> 1);
          float cv = cg[a][b][c];
          if constexpr (WB == 8) {
            cv = fmaf(16.f, ch[a % NH][b][c], cv);
            ch[a % NH][b][c] = 0.f;
          }
          acc[a][b][c] += sj[j] * cv - czj[j] * xo[a][c & 1];
          cg[a][b][c] = 0.f;
        }
#pragma unroll
      for (int c = 0; c < 4; ++c) xo[a][c] = 0.f;
    }
  };
  // fp32 bit pattern of (bias + z) built as z * 2^e + bits(bias): the bias of the codes in the MMA
  // sums is M (4-bit) or M + 16 M (the two nibbles of 8-bit); z * 2^e lands on the units bit of
  // the bias's mantissa (bias 128: 2^16, 1024: 2^13, 2176: 2^12, 17408: 2^9).
  constexpr uint32_t kBiasBits = WB == 8 ? (BF16 ? 0x45080000u : 0x46880000u) : (BF16 ? 0x43000000u : 0x44800000u);
  constexpr uint32_t kZUnit = WB == 8 ? (BF16 ? 4096u : 512u) : (BF16 ? 65536u : 8192u);
  auto load_sz = [&](const uint8_t* srow, const uint8_t* zrow) {
    const uint2 sv = *reinterpret_cast<const uint2*>(srow + cw * 2);
    uint32_t zw = *reinterpret_cast<const uint32_t*>(zrow + (cw * WB / 32) * 4);
    constexpr uint32_t kZMask = (1u << WB) - 1u;
    if (p.v1) {  // (z + 1) mod 2^WB in every field of the word at once
      constexpr uint32_t kLow = WB == 8 ? 0x7F7F7F7Fu : 0x77777777u;
      constexpr uint32_t kOne = WB == 8 ? 0x01010101u : 0x11111111u;
      zw = ((zw & kLow) + kOne) ^ (zw & ~kLow);
    }
    float sc[4];
    if (p.s_dtype == kF16) {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
      sc[0] = a.x; sc[1] = a.y; sc[2] = b.x; sc[3] = b.y;
    } else {
      sc[0] = __uint_as_float(sv.x << 16);
      sc[1] = __uint_as_float(sv.x & 0xFFFF0000u);
      sc[2] = __uint_as_float(sv.y << 16);
      sc[3] = __uint_as_float(sv.y & 0xFFFF0000u);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t z = (zw >> (zsh + WB * j)) & kZMask;
      sj[j] = sc[j];
      // exact for 4-bit codes (<= 19 significant bits); 8-bit: exact for bf16 scales, one
      // fp32 rounding for fp16 scales
      czj[j] = sc[j] * __uint_as_float(z * kZUnit + kBiasBits);
    }
  };

  bool first = true, ok = true;
  int cur_grp = -1;  // group of the warp's last stage when a group spans whole stages
  for (int i = kh; i < nst; i += 2) {
    const int s = i % Cfg::kDepth;
    if (!mbar_wait_ns(&full[s], (i / Cfg::kDepth) & 1, abort_flag, kDevErrWFull, gp.wait_ns)) {
      ok = false;
      break;
    }
    const uint8_t* wst = smem + Cfg::kWOff + s * Cfg::kWBytes + wn * 2048;
    const uint8_t* sst = smem + Cfg::kSOff + s * Cfg::kSBytes;
    const uint8_t* zst = smem + Cfg::kZOff + s * Cfg::kZBytes;
    const uint8_t* xst = smem + Cfg::kXOff + s * Cfg::kXBytes;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // step within the stage
      // group boundaries (warp-uniform)
      bool new_grp;
      int srow;
      if (gp.rows_sz == 1) {
        new_grp = false;
        if (j == 0) {
          const int grp = ((kb0 + i) * KS) / p.gs;
          new_grp = grp != cur_grp;
          cur_grp = grp;
        }
        srow = 0;
      } else {
        new_grp = (j & (spg_step - 1)) == 0;
        srow = j >> spg_shift;
      }
      if (new_grp) {
        if (!first) flush();
        first = false;
        load_sz(sst + srow * (kGemvCols * 2), zst + srow * kZRowBytes);
      }
      const int r = 4 * j + t;  // word row within the slab
      const uint4 w = *reinterpret_cast<const uint4*>(wst + r * 128 + ((g ^ (r & 7)) << 4));
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
      if constexpr (WB == 8) {
        // lane k = KSTEP j + 4t + {0..3}; nibble pairs (lo k0, lo k2), (hi k0, hi k2),
        // (lo k1, lo k3), (hi k1, hi k3) of each column
        uint32_t pr[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          pr[q][0] = lop3_and_or(wv[q], 0x000F000Fu, P::kMagic);
          pr[q][1] = lop3_and_or(wv[q] >> 4, 0x000F000Fu, P::kMagic);
          pr[q][2] = lop3_and_or(wv[q] >> 8, 0x000F000Fu, P::kMagic);
          pr[q][3] = lop3_and_or(wv[q] >> 12, 0x000F000Fu, P::kMagic);
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint2 xv = *reinterpret_cast<const uint2*>(xst + (g + 8 * mt) * (KS * 2) + (KSTEP * j + 4 * t) * 2);
          const uint32_t b0 = prmt(xv.x, xv.y, 0x5410u);  // (x0, x2)
          const uint32_t b1 = prmt(xv.x, xv.y, 0x7632u);  // (x1, x3)
#pragma unroll
          for (int beta = 0; beta < 2; ++beta) {
            const uint32_t alo[4] = {pr[2 * beta][0], pr[2 * beta + 1][0], pr[2 * beta][2], pr[2 * beta + 1][2]};
            const uint32_t ahi[4] = {pr[2 * beta][1], pr[2 * beta + 1][1], pr[2 * beta][3], pr[2 * beta + 1][3]};
            mma_16816<BF16>(cg[mt][beta], alo, b0, b1);
            mma_16816<BF16>(ch[mt % NH][beta], ahi, b0, b1);
          }
          mma_16816<BF16>(xo[mt], ones4, b0, b1);
        }
        continue;
      }
      uint4 xv[MT];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        xv[mt] = *reinterpret_cast<const uint4*>(xst + (g + 8 * mt) * (KS * 2) + (KSTEP * j + 8 * t) * 2);
      uint32_t pr[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pr[q][0] = lop3_and_or(wv[q], 0x000F000Fu, P::kMagic);
        pr[q][1] = lop3_and_or(wv[q] >> 4, 0x000F000Fu, P::kMagic);
        pr[q][2] = lop3_and_or(wv[q] >> 8, 0x000F000Fu, P::kMagic);
        pr[q][3] = lop3_and_or(wv[q] >> 12, 0x000F000Fu, P::kMagic);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t b00, b01, b10, b11;
        x_frags(xv[mt], b00, b01, b10, b11);
#pragma unroll
        for (int beta = 0; beta < 2; ++beta) {
          const uint32_t a0[4] = {pr[2 * beta][0], pr[2 * beta + 1][0], pr[2 * beta][1], pr[2 * beta + 1][1]};
          const uint32_t a1[4] = {pr[2 * beta][2], pr[2 * beta + 1][2], pr[2 * beta][3], pr[2 * beta + 1][3]};
          mma_16816<BF16>(cg[mt][beta], a0, b00, b01);
          mma_16816<BF16>(cg[mt][beta], a1, b10, b11);
        }
        mma_16816<BF16>(xo[mt], ones4, b00, b01);
        mma_16816<BF16>(xo[mt], ones4, b10, b11);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!first) flush();

  // reduce the two k halves of the CTA (named barrier over the 256 consumer threads)
  if (kh == 1) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[wn][lane][a * 8 + b * 4 + c] = acc[a][b][c];
  }
  const bool any_fail = named_bar_or(1, kGtConsumerWarps * 32, !ok);
  if (kh == 0) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] += red[wn][lane][a * 8 + b * 4 + c];
  }
  griddep_wait();  // the previous kernel is done with the workspace and the output
  // a failed CTA (its error is recorded) still takes its split-K ticket and writes nothing
  gemv_finish_n<BF16, MT>(p, acc, kh, col, t, tile, split, &is_last, kGtConsumerWarps * 32, any_fail);
}

}  // namespace oc
