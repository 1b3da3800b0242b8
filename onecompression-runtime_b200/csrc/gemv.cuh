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

struct GemvStage {
  uint4 w;        // 4 words: columns 4g..4g+3 at word row kw
  uint4 xa;       // x[token g][8kw .. 8kw+7]
  uint4 xb;       // x[token g+8][...] (MT == 2)
  uint2 s;        // 4 scales (16-bit each)
  uint32_t z;     // packed zero word
  int valid;
};

// Every lane of a warp must execute the same mma.sync, so out-of-range lanes are not
// skipped: a k-word past K loads zero activations (its B rows contribute nothing), a
// column past N loads zero weights/scales (its A rows feed only discarded outputs) but
// still loads the activations, because a lane's B fragment feeds every row of the tile.
template <int MT>
__device__ __forceinline__ void gemv_load(GemvStage& st, const GemvParams& p, int kw, int col, int g) {
  const int kw_rows = p.Kp >> 3;
  const bool kvalid = kw < kw_rows;
  st.valid = kvalid && (col < p.N);
  st.w = make_uint4(0, 0, 0, 0);
  st.xa = make_uint4(0, 0, 0, 0);
  st.xb = make_uint4(0, 0, 0, 0);
  st.s = make_uint2(0, 0);
  st.z = 0;
  if (!kvalid) return;
  if (g < p.M) st.xa = __ldg(reinterpret_cast<const uint4*>(p.x + (long long)g * p.ldx + 8 * kw));
  if (MT == 2 && g + 8 < p.M) st.xb = __ldg(reinterpret_cast<const uint4*>(p.x + (long long)(g + 8) * p.ldx + 8 * kw));
  if (!st.valid) return;
  st.w = __ldg(reinterpret_cast<const uint4*>(p.qw + (long long)kw * p.N + col));
  const int grp = p.wgrp ? __ldg(p.wgrp + kw) : (8 * kw) / p.gs;
  st.s = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p.s) + (long long)grp * p.N + col));
  st.z = __ldg(p.qz + (long long)grp * (p.N >> 3) + (col >> 3));
}

template <bool BF16, bool HAS_LO, int MT>
__device__ __forceinline__ void gemv_compute(const GemvStage& st, const GemvParams& p, int col,
                                             float (&acc)[MT][2][4]) {
  using P = Pair<BF16>;
  const int zsh = 4 * (col & 7);
  uint32_t pr[4][4];  // [column j][pair: (k0,k4) (k1,k5) (k2,k6) (k3,k7)]
  const uint32_t sw[4] = {st.s.x & 0xFFFFu, st.s.x >> 16, st.s.y & 0xFFFFu, st.s.y >> 16};
  const uint32_t wv[4] = {st.w.x, st.w.y, st.w.z, st.w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t z = (st.z >> (zsh + 4 * j)) & 0xFu;
    if (p.v1) z = (z + 1u) & 0xFu;
    const float s = (p.s_dtype == kF16) ? __half2float(__ushort_as_half((uint16_t)sw[j]))
                                        : __bfloat162float(__ushort_as_bfloat16((uint16_t)sw[j]));
    const DqConst<BF16> c = make_dq_const<BF16>(s, (int)z);
    const uint32_t w = wv[j];
    pr[j][0] = dq_pair<BF16, HAS_LO>(lop3_and_or(w, 0x000F000Fu, P::kMagic), c);
    pr[j][1] = dq_pair<BF16, HAS_LO>(lop3_and_or(w >> 4, 0x000F000Fu, P::kMagic), c);
    pr[j][2] = dq_pair<BF16, HAS_LO>(lop3_and_or(w >> 8, 0x000F000Fu, P::kMagic), c);
    pr[j][3] = dq_pair<BF16, HAS_LO>(lop3_and_or(w >> 12, 0x000F000Fu, P::kMagic), c);
  }
  // B fragments: natural x (x0x1, x2x3, x4x5, x6x7) -> (x0x4, x1x5) and (x2x6, x3x7)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const uint4 xv = (mt == 0) ? st.xa : st.xb;
    const uint32_t b00 = prmt(xv.x, xv.z, 0x5410u);  // (x0, x4)
    const uint32_t b01 = prmt(xv.x, xv.z, 0x7632u);  // (x1, x5)
    const uint32_t b10 = prmt(xv.y, xv.w, 0x5410u);  // (x2, x6)
    const uint32_t b11 = prmt(xv.y, xv.w, 0x7632u);  // (x3, x7)
#pragma unroll
    for (int beta = 0; beta < 2; ++beta) {
      const uint32_t a0[4] = {pr[2 * beta][0], pr[2 * beta + 1][0], pr[2 * beta][1], pr[2 * beta + 1][1]};
      const uint32_t a1[4] = {pr[2 * beta][2], pr[2 * beta + 1][2], pr[2 * beta][3], pr[2 * beta + 1][3]};
      mma_16816<BF16>(acc[mt][beta], a0, b00, b01);
      mma_16816<BF16>(acc[mt][beta], a1, b10, b11);
    }
  }
}

// Split-K partials (deterministic last-CTA reduction), bias, rounding, store.
// fragment -> (token, 4 columns): token 8*a + 2t + h has columns col..col+3 =
// {acc[a][0][h], acc[a][0][2+h], acc[a][1][h], acc[a][1][2+h]}
template <bool BF16, int MT>
__device__ __forceinline__ void gemv_finish(const GemvParams& p, float (&acc)[MT][2][4], int wk, int col, int t,
                                            int tile, int split, int* is_last) {
  if (p.splits > 1) {
    if (wk == 0 && col < p.N) {
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
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(p.tickets + tile, 1u);
      *is_last = (prev == (unsigned)(p.splits - 1));
    }
    __syncthreads();
    if (!*is_last) return;
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
    if (threadIdx.x == 0) p.tickets[tile] = 0u;  // re-arm for the next launch (stream order)
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

template <bool BF16, bool HAS_LO, int MT, int DEPTH>
__global__ void __launch_bounds__(kGemvThreads) gptq_gemv_kernel(const GemvParams p) {
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

  float acc[MT][2][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

  // this warp's steps: step0 + wk, step0 + wk + kGemvWarpsK, ...
  GemvStage buf[DEPTH];
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) {
    const int s = step0 + wk + d * kGemvWarpsK;
    gemv_load<MT>(buf[d], p, s < step1 ? 4 * s + t : 0x7fffffff, col, g);
  }
  for (int base = step0 + wk; base < step1; base += DEPTH * kGemvWarpsK) {
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) {
      const int s = base + d * kGemvWarpsK;
      if (s < step1) gemv_compute<BF16, HAS_LO, MT>(buf[d], p, col, acc);
      const int sn = s + DEPTH * kGemvWarpsK;
      gemv_load<MT>(buf[d], p, sn < step1 ? 4 * sn + t : 0x7fffffff, col, g);
    }
  }

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
// are accumulated together before its correction.
template <bool BF16, int MT, int DEPTH>
__global__ void __launch_bounds__(kGemvThreads) gptq_gemv_fact_kernel(const GemvParams p) {
  using P = Pair<BF16>;
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
  const int steps_per_group = p.gs / 32;
  const uint32_t ones = BF16 ? 0x3F803F80u : 0x3C003C00u;
  const uint32_t ones4[4] = {ones, ones, ones, ones};

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
  int cur_grp = -1;

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

  GemvStage buf[DEPTH];
#pragma unroll
  for (int d = 0; d < DEPTH; ++d) {
    const int s = ws0 + d;
    gemv_load<MT>(buf[d], p, s < ws1 ? 4 * s + t : 0x7fffffff, col, g);
  }
  for (int base = ws0; base < ws1; base += DEPTH) {
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) {
      const int s = base + d;
      if (s < ws1) {  // warp-uniform
        const int grp = s / steps_per_group;
        if (grp != cur_grp) {  // warp-uniform: a 32-k step lies inside one group
          if (cur_grp >= 0) flush();
          const uint32_t sw4[4] = {buf[d].s.x & 0xFFFFu, buf[d].s.x >> 16, buf[d].s.y & 0xFFFFu, buf[d].s.y >> 16};
          const int zsh = 4 * (col & 7);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t z = (buf[d].z >> (zsh + 4 * j)) & 0xFu;
            if (p.v1) z = (z + 1u) & 0xFu;
            const float sv = (p.s_dtype == kF16) ? __half2float(__ushort_as_half((uint16_t)sw4[j]))
                                                 : __bfloat162float(__ushort_as_bfloat16((uint16_t)sw4[j]));
            sj[j] = sv;
            czj[j] = sv * (P::kMagicF + (float)z);   // exact: <= 19 significant bits
          }
          cur_grp = grp;
        }
        const uint32_t wv[4] = {buf[d].w.x, buf[d].w.y, buf[d].w.z, buf[d].w.w};
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
          const uint4 xv = (mt == 0) ? buf[d].xa : buf[d].xb;
          const uint32_t b00 = prmt(xv.x, xv.z, 0x5410u);
          const uint32_t b01 = prmt(xv.x, xv.z, 0x7632u);
          const uint32_t b10 = prmt(xv.y, xv.w, 0x5410u);
          const uint32_t b11 = prmt(xv.y, xv.w, 0x7632u);
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
      const int sn = s + DEPTH;
      gemv_load<MT>(buf[d], p, sn < ws1 ? 4 * sn + t : 0x7fffffff, col, g);
    }
  }
  if (cur_grp >= 0) flush();

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
