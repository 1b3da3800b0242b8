// Decode-sized (M <= 16) split-K GEMV over AutoGPTQ int4 words, HBM-bound.
//
// Replaces the reference's per-call full dequant + F.linear (packed_gptq_linear.py:66-74)
// and the small-M launches of the Triton fused kernel (fused_int4_linear.py:127-272).
//
// Layout trick: Y^T = W * X^T with W as the mma A operand (rows = output
// features n, 16 per mma) and X^T as the B operand (8 tokens per mma).
//   * A warp owns 32 output columns; thread (g = lane/4, t = lane%4) loads one
//     128-bit vector qweight[kw0 + t][n0 + 4g .. 4g+3] per 32-k step: four
//     GPTQ words = 4 columns x 8 k, and a warp load covers four fully used
//     128-byte rows of qweight.
//   * Its 4 columns are rows (g, g+8) of two m16n8k16 tiles (beta = 0, 1).
//   * The 16 k of an mma are a permutation of the 32-k step: thread t supplies
//     the k of word (kw0 + t). lop3 against the magic 128.0 (bf16) / 1024.0
//     (fp16) extracts nibble pairs (i, i+4) of a word directly into a packed
//     pair register, so the B fragment takes x in the matching order
//     [x0 x4 | x1 x5] and [x2 x6 | x3 x7], built with two prmt per pair.
//   * Dequant is exact: w = RNE(s * (q - z)) (see DqConst), i.e. the mma
//     consumes exactly the weights quant_utils.dequant_gptq_to_fp produces.
// Split-K partials go to an fp32 workspace; the last CTA of each column tile
// (atomic ticket) sums them in split order (deterministic), adds the bias
// and writes the output, then re-arms the ticket for the next launch.
#pragma once

#include "common.cuh"

namespace oc {

struct GemvParams {
  const uint16_t* x;        // [M, ldx] activations (already gathered when the layer has a K permutation)
  long long ldx;
  int M;
  const uint32_t* qw;       // [Kp/8, N]
  const uint32_t* qz;       // [G, N/8]
  const void* s;            // [G, N]
  int s_dtype;
  const int32_t* wgrp;      // [Kp/8] group of each word, or null: group = 8*kw / gs
  int Kp, N, G, gs, v1;
  const void* bias;         // [N] or null
  int bias_dtype;
  const uint16_t* residual; // optional [M, ldr] added after the activation
  long long ldr;
  int act;                  // Act
  uint16_t* out;            // [M, ldc]
  long long ldc;
  float* ws;                // [splits, M, N] fp32 partials (splits > 1)
  unsigned* tickets;        // [ceil(N/128)] zero-initialised, self re-arming
  int splits;
  int kstep_per_split;      // 32-k steps per split
};

constexpr int kGemvWarpsN = 4;        // 4 x 32 = 128 columns per CTA
constexpr int kGemvWarpsK = 2;
constexpr int kGemvThreads = 32 * kGemvWarpsN * kGemvWarpsK;
constexpr int kGemvCols = 32 * kGemvWarpsN;

template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if (BF16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// ---- per-warp cp.async ring --------------------------------------------------------------
// Each warp streams its K range through a ring of kGemvDepth<MT> shared-memory slots filled
// with cp.async (16-byte weight vectors straight to shared memory, no register staging), so a
// warp keeps up to depth x 512 bytes of packed weights in flight. Every lane reads back only
// the bytes it loaded itself, so a lane's own cp.async.wait_group is the only synchronisation.
// Slot layout (structure of arrays, conflict-free 16/8/4-byte lane accesses):
//   w[32] uint4 | x[MT][32] uint4 | s[32] uint2 | z[32] uint32
template <int MT> struct GemvRing {
  static constexpr int kDepth = MT == 1 ? 8 : 6;
  static constexpr int kSlotBytes = 32 * 16 + MT * 32 * 16 + 32 * 8 + 32 * 4;
  static constexpr int kWarpBytes = kDepth * kSlotBytes;
  static constexpr int kSmemBytes = kGemvThreads / 32 * kWarpBytes;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Issue the loads of 32-k step `s` (word kw = 4s + t of this lane) into ring slot `slot`.
// Out-of-range words/columns are zero-filled; a column past N still loads the activations,
// because every lane's B fragment feeds every row of the tile. Scales/zeros are loaded only
// when `need_sz` (a group starts at this step, or per-word groups).
template <int MT>
__device__ __forceinline__ void gemv_issue(uint8_t* slot, const GemvParams& p, int s, int step1, int col, int g, int t,
                                           int lane, bool need_sz) {
  const int kw = 4 * s + t;
  const bool kvalid = s < step1 && kw < (p.Kp >> 3);
  const bool valid = kvalid && col < p.N;
  const int kwc = kvalid ? kw : 0;
  const int colc = col < p.N ? col : 0;
  cp_async16(slot + lane * 16, p.qw + (long long)kwc * p.N + colc, valid);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int tok = g + 8 * mt;
    if (tok < p.M) cp_async16(slot + 512 + mt * 512 + lane * 16, p.x + (long long)tok * p.ldx + 8 * kwc, kvalid);
  }
  if (need_sz) {
    const int grp = valid ? (p.wgrp ? __ldg(p.wgrp + kw) : (8 * kw) / p.gs) : 0;
    cp_async8(slot + 512 + MT * 512 + lane * 8,
              reinterpret_cast<const uint16_t*>(p.s) + (long long)grp * p.N + colc, valid);
    cp_async4(slot + 512 + MT * 512 + 256 + lane * 4, p.qz + (long long)grp * (p.N >> 3) + (colc >> 3), valid);
  }
}

template <int MT>
__device__ __forceinline__ void gemv_read_x(const uint8_t* slot, const GemvParams& p, int g, int lane,
                                            uint4 (&xv)[MT]) {
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
    xv[mt] = (g + 8 * mt < p.M) ? *reinterpret_cast<const uint4*>(slot + 512 + mt * 512 + lane * 16)
                                : make_uint4(0, 0, 0, 0);
}

// B fragments: natural x (x0x1, x2x3, x4x5, x6x7) -> (x0x4, x1x5) and (x2x6, x3x7)
__device__ __forceinline__ void x_frags(const uint4& xv, uint32_t& b00, uint32_t& b01, uint32_t& b10, uint32_t& b11) {
  b00 = prmt(xv.x, xv.z, 0x5410u);
  b01 = prmt(xv.x, xv.z, 0x7632u);
  b10 = prmt(xv.y, xv.w, 0x5410u);
  b11 = prmt(xv.y, xv.w, 0x7632u);
}

// Split-K partials (deterministic last-CTA reduction), bias, rounding, store.
// fragment -> (token, 4 columns): token 8*a + 2t + h has columns col..col+3 =
// {acc[a][0][h], acc[a][0][2+h], acc[a][1][h], acc[a][1][2+h]}
// bar_threads = 0: the whole CTA takes part (__syncthreads); otherwise the first bar_threads
// threads do, synchronised on named barrier 2 (kernels whose producer warp has left).
__device__ __forceinline__ void gemv_bar(int bar_threads) {
  if (bar_threads == 0)
    __syncthreads();
  else
    named_bar_sync(2, bar_threads);
}

// Ticket word of a column tile: arrivals in the low 16 bits, arrivals of CTAs that failed (a
// bounded wait gave up) from bit 16. Failing CTAs still take their ticket, so the last CTA always
// re-arms it and the tickets are zero after every launch, failed or not; the output of a tile
// with a failed split is left unwritten (the error word tells the host).
constexpr unsigned kTicketFail = 1u << 16;

template <bool BF16, int MT>
__device__ __forceinline__ void gemv_finish_n(const GemvParams& p, float (&acc)[MT][2][4], int wk, int col, int t,
                                              int tile, int split, int* is_last, int bar_threads,
                                              bool failed = false) {
  if (p.splits > 1) {
    if (!failed && wk == 0 && col < p.N) {
#pragma unroll
      for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = 8 * a + 2 * t + h;
          if (tok < p.M) {
            const float4 v = make_float4(acc[a][0][h], acc[a][0][2 + h], acc[a][1][h], acc[a][1][2 + h]);
            *reinterpret_cast<float4*>(p.ws + ((long long)split * p.M + tok) * p.N + col) = v;
          }
        }
    }
    __threadfence();
    gemv_bar(bar_threads);
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.tickets + tile, failed ? 1u + kTicketFail : 1u);
      const bool last = (prev & (kTicketFail - 1u)) == (unsigned)(p.splits - 1);
      *is_last = !last ? 0 : ((prev >= kTicketFail || failed) ? 2 : 1);
      if (last) p.tickets[tile] = 0u;  // re-arm for the next launch (stream order)
    }
    gemv_bar(bar_threads);
    if (*is_last != 1) return;
    __threadfence();
    if (wk == 0 && col < p.N) {
#pragma unroll
      for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = 8 * a + 2 * t + h;
          if (tok < p.M) {
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sp = 0; sp < p.splits; ++sp) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(p.ws + ((long long)sp * p.M + tok) * p.N + col));
              sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
            }
            acc[a][0][h] = sum.x; acc[a][0][2 + h] = sum.y; acc[a][1][h] = sum.z; acc[a][1][2 + h] = sum.w;
          }
        }
    }
  } else if (failed) {
    return;
  }
  if (wk != 0 || col >= p.N) return;
  float bv[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bv[j] = load_as_f32(p.bias, p.bias_dtype, col + j);
  }
  const int odt = BF16 ? kBF16 : kF16;
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tok = 8 * a + 2 * t + h;
      if (tok < p.M) {
        const uint16_t* res = p.residual ? p.residual + (long long)tok * p.ldr + col : nullptr;
        const uint16_t o0 = f32_to_bits(epilogue_value(acc[a][0][h], bv[0], p.act, res, odt), odt);
        const uint16_t o1 = f32_to_bits(epilogue_value(acc[a][0][2 + h], bv[1], p.act, res ? res + 1 : res, odt), odt);
        const uint16_t o2 = f32_to_bits(epilogue_value(acc[a][1][h], bv[2], p.act, res ? res + 2 : res, odt), odt);
        const uint16_t o3 = f32_to_bits(epilogue_value(acc[a][1][2 + h], bv[3], p.act, res ? res + 3 : res, odt), odt);
        uint16_t* dst = p.out + (long long)tok * p.ldc + col;
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack2(o0, o1), pack2(o2, o3));
      }
    }
}

// Exact-weight GEMV (any group structure, incl. per-word group tables): every weight is
// dequantized to RNE(s (q - z)) in the activation type before the MMA.
template <bool BF16, int MT>
__device__ __forceinline__ void gemv_finish(const GemvParams& p, float (&acc)[MT][2][4], int wk, int col, int t,
                                            int tile, int split, int* is_last) {
  gemv_finish_n<BF16, MT>(p, acc, wk, col, t, tile, split, is_last, 0);
}

template <bool BF16, bool HAS_LO, int MT>
__global__ void __launch_bounds__(kGemvThreads) gptq_gemv_kernel(const GemvParams p) {
  using P = Pair<BF16>;
  using Ring = GemvRing<MT>;
  extern __shared__ __align__(128) uint8_t gemv_smem[];
  __shared__ float red[kGemvWarpsN][32][MT * 8];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp % kGemvWarpsN, wk = warp / kGemvWarpsN;
  const int g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int col = tile * kGemvCols + wn * 32 + 4 * g;
  const int total_steps = (p.Kp + 31) / 32;
  const int step0 = split * p.kstep_per_split;
  const int step1 = min(total_steps, step0 + p.kstep_per_split);
  const int half = (step1 - step0 + kGemvWarpsK - 1) / kGemvWarpsK;
  const int ws0 = step0 + wk * half;
  const int ws1 = min(step1, ws0 + half);
  uint8_t* ring = gemv_smem + warp * Ring::kWarpBytes;

  float acc[MT][2][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

#pragma unroll
  for (int d = 0; d < Ring::kDepth; ++d) {
    gemv_issue<MT>(ring + d * Ring::kSlotBytes, p, ws0 + d, ws1, col, g, t, lane, true);
    cp_async_commit();
  }
  const int zsh = 4 * (col & 7);
  int slot_i = 0;
  for (int s = ws0; s < ws1; ++s) {
    cp_async_wait<Ring::kDepth - 1>();
    uint8_t* slot = ring + slot_i * Ring::kSlotBytes;
    const uint4 w = *reinterpret_cast<const uint4*>(slot + lane * 16);
    const uint2 sv = *reinterpret_cast<const uint2*>(slot + 512 + MT * 512 + lane * 8);
    const uint32_t zw = *reinterpret_cast<const uint32_t*>(slot + 512 + MT * 512 + 256 + lane * 4);
    uint4 xv[MT];
    gemv_read_x<MT>(slot, p, g, lane, xv);
    gemv_issue<MT>(slot, p, s + Ring::kDepth, ws1, col, g, t, lane, true);
    cp_async_commit();
    if (++slot_i == Ring::kDepth) slot_i = 0;

    uint32_t pr[4][4];  // [column j][pair: (k0,k4) (k1,k5) (k2,k6) (k3,k7)]
    const uint32_t sw[4] = {sv.x & 0xFFFFu, sv.x >> 16, sv.y & 0xFFFFu, sv.y >> 16};
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t z = (zw >> (zsh + 4 * j)) & 0xFu;
      if (p.v1) z = (z + 1u) & 0xFu;
      const float sc = (p.s_dtype == kF16) ? __half2float(__ushort_as_half((uint16_t)sw[j]))
                                           : __bfloat162float(__ushort_as_bfloat16((uint16_t)sw[j]));
      const DqConst<BF16> c = make_dq_const<BF16>(sc, (int)z);
      pr[j][0] = dq_pair<BF16, HAS_LO>(lop3_and_or(wv[j], 0x000F000Fu, P::kMagic), c);
      pr[j][1] = dq_pair<BF16, HAS_LO>(lop3_and_or(wv[j] >> 4, 0x000F000Fu, P::kMagic), c);
      pr[j][2] = dq_pair<BF16, HAS_LO>(lop3_and_or(wv[j] >> 8, 0x000F000Fu, P::kMagic), c);
      pr[j][3] = dq_pair<BF16, HAS_LO>(lop3_and_or(wv[j] >> 12, 0x000F000Fu, P::kMagic), c);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      uint32_t b00, b01, b10, b11;
      x_frags(xv[mt], b00, b01, b10, b11);
#pragma unroll
      for (int beta = 0; beta < 2; ++beta) {
        const uint32_t a0[4] = {pr[2 * beta][0], pr[2 * beta + 1][0], pr[2 * beta][1], pr[2 * beta + 1][1]};
        const uint32_t a1[4] = {pr[2 * beta][2], pr[2 * beta + 1][2], pr[2 * beta][3], pr[2 * beta + 1][3]};
        mma_16816<BF16>(acc[mt][beta], a0, b00, b01);
        mma_16816<BF16>(acc[mt][beta], a1, b10, b11);
      }
    }
  }
  cp_async_wait<0>();

  // reduce the K-warps of this CTA
  if (wk == 1) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[wn][lane][a * 8 + b * 4 + c] = acc[a][b][c];
  }
  __syncthreads();
  if (wk == 0) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] += red[wn][lane][a * 8 + b * 4 + c];
  }
  gemv_finish<BF16, MT>(p, acc, wk, col, t, tile, split, &is_last);
}

// ------------------------------------------------------------------------------------------
// Factored GEMV for uniform groups spanning whole 32-k steps (gs % 32 == 0, no word table):
// the tensor cores multiply the raw magic-biased codes (M + q) -- exact in bf16/fp16 -- and
// the scale/zero are applied once per group to fp32 sums:
//     sum_k x_k s (q_k - z) = s * sum_k x_k (M + q_k)  -  s (M + z) * sum_k x_k
// sum_k x_k comes from a second MMA against an all-ones A fragment, already in the layout
// of the accumulators. Per weight this leaves only the nibble extraction (lop3 + shift) on
// the CUDA cores; the result is the exact-weight product evaluated in fp32 (it does not
// round the weights to 16 bits first). Warps take contiguous K ranges so a group's steps
// are accumulated together before its correction; scales/zeros are fetched once per group.
template <bool BF16, int MT>
__global__ void __launch_bounds__(kGemvThreads) gptq_gemv_fact_kernel(const GemvParams p) {
  using P = Pair<BF16>;
  using Ring = GemvRing<MT>;
  extern __shared__ __align__(128) uint8_t gemv_smem[];
  __shared__ float red[kGemvWarpsN][32][MT * 8];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wn = warp % kGemvWarpsN, wk = warp / kGemvWarpsN;
  const int g = lane >> 2, t = lane & 3;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int col = tile * kGemvCols + wn * 32 + 4 * g;
  const int total_steps = (p.Kp + 31) / 32;
  const int step0 = split * p.kstep_per_split;
  const int step1 = min(total_steps, step0 + p.kstep_per_split);
  const int half = (step1 - step0 + kGemvWarpsK - 1) / kGemvWarpsK;
  const int ws0 = step0 + wk * half;
  const int ws1 = min(step1, ws0 + half);
  const int spg = p.gs / 32;  // steps per group
  uint8_t* ring = gemv_smem + warp * Ring::kWarpBytes;
  const uint32_t ones = BF16 ? 0x3F803F80u : 0x3C003C00u;
  const uint32_t ones4[4] = {ones, ones, ones, ones};

  // Load-side cursors (step `si`, D steps ahead of the math): running pointers instead of
  // per-step index arithmetic; a group countdown instead of divisions.
  const bool cvalid = col < p.N;
  const int colc = cvalid ? col : 0;
  const int kw_rows = p.Kp >> 3;
  const long long wstride = 4LL * p.N;  // one 32-k step of qweight rows
  const uint32_t* wp = p.qw + (long long)(4 * ws0 + t) * p.N + colc;
  const uint16_t* xp[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) xp[mt] = p.x + (long long)min(g + 8 * mt, p.M - 1) * p.ldx + 8 * (4 * ws0 + t);
  int grp_i = ws0 / spg;
  int left_i = spg - (ws0 - grp_i * spg);  // steps of the current group left, counting si
  const uint16_t* sp = reinterpret_cast<const uint16_t*>(p.s) + (long long)grp_i * p.N + colc;
  const uint32_t* zp = p.qz + (long long)grp_i * (p.N >> 3) + (colc >> 3);
  int si = ws0;
  auto issue = [&](uint8_t* slot, bool need_sz) {
    const bool kvalid = si < ws1 && 4 * si + t < kw_rows;
    cp_async16(slot + lane * 16, kvalid ? (const void*)wp : (const void*)p.qw, kvalid && cvalid);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
      if (g + 8 * mt < p.M) cp_async16(slot + 512 + mt * 512 + lane * 16, kvalid ? (const void*)xp[mt] : (const void*)p.x, kvalid);
    if (need_sz) {
      const bool v = kvalid && cvalid;
      cp_async8(slot + 512 + MT * 512 + lane * 8, v ? (const void*)sp : p.s, v);
      cp_async4(slot + 512 + MT * 512 + 256 + lane * 4, v ? (const void*)zp : (const void*)p.qz, v);
    }
    cp_async_commit();
    ++si;
    wp += wstride;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) xp[mt] += 32;
    if (--left_i == 0) {
      left_i = spg;
      sp += p.N;
      zp += p.N >> 3;
    }
  };

  float acc[MT][2][4], cg[MT][2][4], xo[MT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a) {
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = cg[a][b][c] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) xo[a][c] = 0.f;
  }
  float sj[4] = {0.f, 0.f, 0.f, 0.f}, czj[4] = {0.f, 0.f, 0.f, 0.f};

  auto flush = [&]() {
#pragma unroll
    for (int a = 0; a < MT; ++a) {
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = 2 * b + (c >> 1);
          acc[a][b][c] += sj[j] * cg[a][b][c] - czj[j] * xo[a][c & 1];
          cg[a][b][c] = 0.f;
        }
#pragma unroll
      for (int c = 0; c < 4; ++c) xo[a][c] = 0.f;
    }
  };

#pragma unroll
  for (int d = 0; d < Ring::kDepth; ++d) issue(ring + d * Ring::kSlotBytes, d == 0 || left_i == spg);
  const int zsh = 4 * (col & 7);
  int slot_i = 0;
  int left_c = spg - (ws0 - (ws0 / spg) * spg);  // math side: steps left in the current group
  bool first = true;
  for (int s = ws0; s < ws1; ++s) {
    cp_async_wait<Ring::kDepth - 1>();
    uint8_t* slot = ring + slot_i * Ring::kSlotBytes;
    const uint4 w = *reinterpret_cast<const uint4*>(slot + lane * 16);
    uint4 xv[MT];
    gemv_read_x<MT>(slot, p, g, lane, xv);
    if (first || left_c == spg) {  // warp-uniform: a group starts (or the range does)
      if (!first) flush();
      first = false;
      const uint2 sv = *reinterpret_cast<const uint2*>(slot + 512 + MT * 512 + lane * 8);
      const uint32_t zw = *reinterpret_cast<const uint32_t*>(slot + 512 + MT * 512 + 256 + lane * 4);
      const uint32_t sw4[4] = {sv.x & 0xFFFFu, sv.x >> 16, sv.y & 0xFFFFu, sv.y >> 16};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t z = (zw >> (zsh + 4 * j)) & 0xFu;
        if (p.v1) z = (z + 1u) & 0xFu;
        const float sc = (p.s_dtype == kF16) ? __half2float(__ushort_as_half((uint16_t)sw4[j]))
                                             : __bfloat162float(__ushort_as_bfloat16((uint16_t)sw4[j]));
        sj[j] = sc;
        czj[j] = sc * (P::kMagicF + (float)z);  // exact: <= 19 significant bits
      }
    }
    if (--left_c == 0) left_c = spg;
    issue(slot, left_i == spg);
    if (++slot_i == Ring::kDepth) slot_i = 0;

    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
    uint32_t pr[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pr[j][0] = lop3_and_or(wv[j], 0x000F000Fu, P::kMagic);
      pr[j][1] = lop3_and_or(wv[j] >> 4, 0x000F000Fu, P::kMagic);
      pr[j][2] = lop3_and_or(wv[j] >> 8, 0x000F000Fu, P::kMagic);
      pr[j][3] = lop3_and_or(wv[j] >> 12, 0x000F000Fu, P::kMagic);
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
  if (!first) flush();
  cp_async_wait<0>();

  // ---- reduction across the K warps, split-K, epilogue (same as gptq_gemv_kernel)
  if (wk == 1) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[wn][lane][a * 8 + b * 4 + c] = acc[a][b][c];
  }
  __syncthreads();
  if (wk == 0) {
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] += red[wn][lane][a * 8 + b * 4 + c];
  }
  gemv_finish<BF16, MT>(p, acc, wk, col, t, tile, split, &is_last);
}

}  // namespace oc
