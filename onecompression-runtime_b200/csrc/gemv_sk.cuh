// Decode-sized (M <= 8) stream-K GEMV over AutoGPTQ int4 words (OC_OPT_GEMV_IMPL = 3), for layers
// with uniform groups of 32, 64 or a multiple of 128 rows and at least 256 columns.
//
// Replaces the reference's per-call dequant + F.linear of PackedGPTQLinear
// (packed_gptq_linear.py:66-74) at decode sizes, act-order included.
//
// Work split. The layer is cut into units of one 256-column tile x 128 k (16 GPTQ word rows,
// 16 KB of codes). Units are numbered tile-major and every CTA takes an equal run of them
// (stream-K, two CTAs per SM), so all SMs stream the same number of bytes whatever the layer
// shape. A run covers the tail of one tile and the head of the next; each (tile, CTA) piece is a
// "segment". A tile covered by one segment is written straight from registers; otherwise every
// segment writes its fp32 partial to the workspace (slot tile + CTA index, unique because runs are
// ordered), takes the tile's ticket, and the last to arrive sums the partials in CTA order
// (deterministic), adds bias / activation / residual, writes the output and re-arms the ticket.
// Tickets are per (tile, consumer warp): each warp owns its 32 columns, writes its partials as it
// goes and takes its tickets at the end of its run, so no warp waits for another mid-run.
//
// Activations. After griddepcontrol.wait (the previous kernel wrote x), the 8 consumer warps
// gather the activation columns of their run into shared memory themselves: through the layer's
// K permutation (act-order; no separate gather kernel) or contiguously. The gathered values are
// stored already in MMA B-fragment order, and the per-group sums sum_k x[m, k] that the factored
// scaling needs are computed in the same pass (warp shuffles), so the main loop issues no
// tensor-core work for them. The act-order indices of the first gather are loaded before the wait.
// A run whose activations exceed the 24 KB fragment buffer is processed in pieces.
//
// Streaming. The producer warp fills the ring's first stages at once; after the consumers' first
// gather its 32 lanes issue TMA L2 prefetches for the rest of the run, so the whole layer is
// requested from HBM early and the later ring loads hit L2.
//
// Arithmetic (as gptq_gemv_tma_kernel): Y^T = W X^T on mma.sync.m16n8k16 with the raw magic-biased
// codes (Mg + q) as A and x as B; per group, s * (C - (Mg + z) * sum_k x) in fp32.
//
// Measured on the config-2 layer set (B200): equal to the split-K kernel at M = 1, slower at M = 4
// (the per-CTA activation gather queues behind the weight stream); the consumers are bound by the
// integer pipe (nibble extraction, ~0.19 warp instructions per weight byte). Not the default.
//
// Roles: warp 8 = TMA producer (lane 0: eight 32-column weight slabs with the 128-byte swizzle,
// the unit's scale and zero rows, per unit into a 4-deep mbarrier ring); warps 0-7 = consumers,
// warp w owns columns [32 w, 32 w + 32) of the tile. Every mbarrier wait is bounded; a warp whose
// wait ran out records the error, still takes its tickets (flagged) and writes nothing.
#pragma once

#include "common.cuh"
#include "gemv.cuh"
#include "gemv_tma.cuh"  // griddep_wait / griddep_launch_dependents

namespace oc {

constexpr int kSkWarps = 8;                        // consumer warps, one per 32-column slab
constexpr int kSkCols = 32 * kSkWarps;             // 256 columns per tile
constexpr int kSkThreads = 32 * (kSkWarps + 1);
constexpr int kSkBK = 128;                         // k per unit: 16 word rows, 4 MMA steps
constexpr int kSkDepth = 4;
constexpr int kSkWBytes = kSkWarps * 16 * 128;     // 8 slabs x [16 rows][32 words], 128B-swizzled
constexpr int kSkSBytes = 4 * kSkCols * 2;         // up to 4 scale rows (groups of 32)
constexpr int kSkZBytes = 4 * (kSkCols / 8) * 4;   // up to 4 rows of packed zeros
constexpr int kSkXBytes = 24576;                   // activation fragments of one piece
constexpr int kSkSumBytes = 2048;                  // per-group activation sums of one piece
constexpr int kSkWOff = 0;
constexpr int kSkSOff = kSkWOff + kSkDepth * kSkWBytes;
constexpr int kSkZOff = kSkSOff + kSkDepth * kSkSBytes;
constexpr int kSkXOff = kSkZOff + kSkDepth * kSkZBytes;
constexpr int kSkSumOff = kSkXOff + kSkXBytes;
constexpr int kSkBarOff = kSkSumOff + kSkSumBytes;
constexpr int kSkSmemBytes = kSkBarOff + (2 * kSkDepth + 1) * 8 + 16 + 1024 /*align*/;
static_assert(kSkSmemBytes <= 113 * 1024, "two CTAs must fit one SM");

struct SkParams {
  const uint16_t* x;        // [M, ldx] activations in the caller's K order
  long long ldx;
  int M;
  const int32_t* kperm;     // [Kp] source column of each kernel-order k (-1: padding), or null
  int K_in;                 // columns of x
  int Kp, N, gs, v1, s_dtype;
  int rows_sz;              // scale/zero rows per unit: 128 / gs for gs < 128, else 1
  int KB;                   // units per tile along K
  int units;                // tiles x KB
  int upc;                  // units per CTA
  const void* bias;
  int bias_dtype;
  const uint16_t* residual;
  long long ldr;
  int act;
  uint16_t* out;
  long long ldc;
  float* ws;                // [tiles + grid][M][256] fp32 partials of tiles split over CTAs
  unsigned* tickets;        // [tiles][8 warps], zero-initialised, self re-arming
  unsigned long long wait_ns;
  int stall_stage;          // failure test only: > 0 leaves unit stall_stage - 1 of CTA 0 unissued
};

// Units of activation fragments one piece holds: 128 k x M tokens x 2 bytes per unit.
__host__ __device__ constexpr int sk_units_per_piece(int M) {
  return kSkXBytes / (256 * M) > 0 ? kSkXBytes / (256 * M) : 1;
}

template <bool BF16>
__device__ __forceinline__ float sk_to_f32(uint32_t b) {
  if constexpr (BF16) return __uint_as_float(b << 16);
  else return __half2float(__ushort_as_half((uint16_t)b));
}

// Kernel-order k of word row `row` of a piece starting at K stage kb0 (row = 16 unit + r).
__device__ __forceinline__ int sk_row_k(int kb0, int row) { return (kb0 + (row >> 4)) * kSkBK + 8 * (row & 15); }

// Act-order source columns of the 8 k of word row `row` (-1 outside the layer).
__device__ __forceinline__ void sk_load_idx(const SkParams& p, int kb0, int rows, int row, int (&src)[8]) {
  const int k0 = sk_row_k(kb0, row);
  if (row < rows && k0 < p.Kp) {
    const int4 a = __ldg(reinterpret_cast<const int4*>(p.kperm + k0));
    const int4 b = __ldg(reinterpret_cast<const int4*>(p.kperm + k0 + 4));
    src[0] = a.x; src[1] = a.y; src[2] = a.z; src[3] = a.w;
    src[4] = b.x; src[5] = b.y; src[6] = b.z; src[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) src[i] = -1;
  }
}

// Gather the activations of the `npu` units starting at K stage `kb0` of a tile into fragment
// order, with their per-flush-group sums. Fragment of (unit pi, word row r = 4 j + t, token m):
// uint4 at index ((pi * 4 + j) * 4 + t) * M + m = { (x0, x4), (x1, x5), (x2, x6), (x3, x7) } of
// k = 128 kb + 8 r + {0..7}. Sums: float at (pi * subs + r / rpf) * M + m, rpf = word rows per
// flush group. Run by the 256 consumer threads (tid 0..255), all of them the same number of
// times; word rows are spread one per thread, so the rpf rows of a flush group sit in rpf
// consecutive lanes. `pre` holds the act-order indices of rows tid and tid + 256 when `npre` > 0.
template <bool BF16>
__device__ __forceinline__ void sk_gather(const SkParams& p, int kb0, int npu, int rpf, uint4* xr, float* sums,
                                          int tid, const int (&pre)[2][8], int npre) {
  const int subs = 16 / rpf;
  const int rows = npu * 16;
  for (int round = 0, base = 0; base < rows; ++round, base += 256) {
    const int row = base + tid;
    const bool valid = row < rows;
    const int pi = row >> 4, r = row & 15;
    const int k0 = sk_row_k(kb0, row);
    const bool kin = valid && k0 < p.Kp;
    int src[8];
    if (p.kperm) {
      if (round < npre) {
#pragma unroll
        for (int i = 0; i < 8; ++i) src[i] = pre[round & 1][i];
      } else {
        sk_load_idx(p, kb0, rows, row, src);
      }
    }
    // tokens in batches of 4: every load of a batch is in flight before the first is used
    for (int m0 = 0; m0 < p.M; m0 += 4) {
      uint32_t v[4][8];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int m = m0 + b;
        const uint16_t* xrow = p.x + (long long)m * p.ldx;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[b][i] = 0u;
        if (kin && m < p.M) {
          if (p.kperm) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (src[i] >= 0 && src[i] < p.K_in) v[b][i] = xrow[src[i]];
          } else if (k0 + 8 <= p.K_in) {
            const uint4 q = *reinterpret_cast<const uint4*>(xrow + k0);
            v[b][0] = q.x & 0xFFFFu; v[b][1] = q.x >> 16; v[b][2] = q.y & 0xFFFFu; v[b][3] = q.y >> 16;
            v[b][4] = q.z & 0xFFFFu; v[b][5] = q.z >> 16; v[b][6] = q.w & 0xFFFFu; v[b][7] = q.w >> 16;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (k0 + i < p.K_in) v[b][i] = xrow[k0 + i];
          }
        }
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int m = m0 + b;
        if (m >= p.M) break;  // uniform: M is the same in every lane
        if (valid)
          xr[((pi * 4 + (r >> 2)) * 4 + (r & 3)) * p.M + m] =
              make_uint4(v[b][0] | (v[b][4] << 16), v[b][1] | (v[b][5] << 16), v[b][2] | (v[b][6] << 16),
                         v[b][3] | (v[b][7] << 16));
        float sm = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) sm += sk_to_f32<BF16>(v[b][i]);
        for (int o = 1; o < rpf; o <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        if (valid && (r & (rpf - 1)) == 0) sums[(pi * subs + r / rpf) * p.M + m] = sm;
      }
    }
  }
}

// out[m, col .. col + 3] for this thread's tokens: epilogue of the four columns' fp32 sums.
template <bool BF16, int MT>
__device__ __forceinline__ void sk_write_out(const SkParams& p, const float (&acc)[MT][2][4], int col, int t) {
  constexpr int odt = BF16 ? kBF16 : kF16;
  float bv[4] = {0.f, 0.f, 0.f, 0.f};
  if (p.bias) {
#pragma unroll
    for (int q = 0; q < 4; ++q) bv[q] = load_as_f32(p.bias, p.bias_dtype, col + q);
  }
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = 8 * a + 2 * t + h;
      if (m < p.M) {
        const uint16_t* res = p.residual ? p.residual + (long long)m * p.ldr + col : nullptr;
        const uint16_t o0 = f32_to_bits(epilogue_value(acc[a][0][h], bv[0], p.act, res, odt), odt);
        const uint16_t o1 = f32_to_bits(epilogue_value(acc[a][0][2 + h], bv[1], p.act, res ? res + 1 : res, odt), odt);
        const uint16_t o2 = f32_to_bits(epilogue_value(acc[a][1][h], bv[2], p.act, res ? res + 2 : res, odt), odt);
        const uint16_t o3 = f32_to_bits(epilogue_value(acc[a][1][2 + h], bv[3], p.act, res ? res + 3 : res, odt), odt);
        *reinterpret_cast<uint2*>(p.out + (long long)m * p.ldc + col) = make_uint2(pack2(o0, o1), pack2(o2, o3));
      }
    }
}

// SPF: MMA steps (32 k) per flush group, 1 / 2 / 4 for groups of 32 / 64 / >= 128 rows, a
// template parameter so the unrolled step loop carries no run-time group tests.
template <bool BF16, int MT, int SPF>
__global__ void __launch_bounds__(kSkThreads, 2)
    gptq_gemv_sk_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_s,
                        const __grid_constant__ CUtensorMap tmap_z, const __grid_constant__ CUtensorMap tmap_pw,
                        const SkParams p) {
  using P = Pair<BF16>;
  extern __shared__ __align__(1024) uint8_t sk_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sk_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSkBarOff);
  uint64_t* empty = full + kSkDepth;
  uint64_t* gathered = empty + kSkDepth;  // the consumers' first activation gather is done
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gathered + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = blockIdx.x * p.upc;
  const int u1 = min(p.units, u0 + p.upc);
  const int nu = u1 - u0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSkDepth; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSkWarps);
    }
    mbar_init(gathered, kSkWarps);
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  griddep_launch_dependents();

  if (warp == kSkWarps) {
    // ------------------------------------------------------------------ producer
    // Weights, scales and zeros are static: requested without waiting for the previous kernel.
    // Lane 0 fills the ring's first stages at once; the L2 prefetch of the rest of the run (all
    // lanes) follows once the consumers have gathered their activations, so those few latency-bound
    // loads are not queued behind the run's whole weight traffic (the first stages of all CTAs
    // already keep HBM busy meanwhile).
    const uint32_t bytes = kSkWBytes + p.rows_sz * (kSkCols * 2 + kSkCols / 2);
    const int stall = blockIdx.x == 0 ? p.stall_stage - 1 : -1;
    int armed[kSkDepth];
#pragma unroll
    for (int i = 0; i < kSkDepth; ++i) armed[i] = -1;
    auto issue = [&](int i) {
      const int s = i % kSkDepth;
      const int u = u0 + i;
      const int tile = u / p.KB, kb = u - tile * p.KB;
      const int col0 = tile * kSkCols;
      mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
      for (int c = 0; c < kSkWarps; ++c)
        tma_load_2d(smem + kSkWOff + s * kSkWBytes + c * 2048, &tmap_w, &full[s], col0 + 32 * c, kb * 16);
      const int g0 = (kb * kSkBK) / p.gs;
      tma_load_2d(smem + kSkSOff + s * kSkSBytes, &tmap_s, &full[s], col0, g0);
      tma_load_2d(smem + kSkZOff + s * kSkZBytes, &tmap_z, &full[s], col0 / 8, g0);
      armed[s] = (i / kSkDepth) & 1;
    };
    const int first = nu < kSkDepth ? nu : kSkDepth;
    if (lane == 0) {
      for (int i = 0; i < first; ++i)
        if (i != stall) issue(i);
    }
    const bool go = mbar_wait_ns(gathered, 0, abort_flag, kDevErrWEmpty, p.wait_ns);
    if (go) {
      for (int i = first + lane; i < nu; i += 32) {
        const int u = u0 + i;
        const int tile = u / p.KB, kb = u - tile * p.KB;
        const int g0 = (kb * kSkBK) / p.gs;
        tma_prefetch_l2_2d(&tmap_pw, tile * kSkCols, kb * 16);
        if (i == first || kb == 0 || g0 != ((kb - 1) * kSkBK) / p.gs) {
          tma_prefetch_l2_2d(&tmap_s, tile * kSkCols, g0);
          tma_prefetch_l2_2d(&tmap_z, tile * kSkCols / 8, g0);
        }
      }
    }
    if (lane == 0) {
      for (int i = first; go && i < nu; ++i) {
        const int s = i % kSkDepth;
        if (!mbar_wait_ns(&empty[s], ((i / kSkDepth) & 1) ^ 1, abort_flag, kDevErrWEmpty, p.wait_ns)) break;
        if (i != stall) issue(i);
      }
      // no bulk copy may be in flight when the CTA exits
#pragma unroll
      for (int s = 0; s < kSkDepth; ++s)
        if (armed[s] >= 0) mbar_drain(&full[s], armed[s]);
    }
    return;  // the producer takes no part in the consumers' named barriers
  }

  // -------------------------------------------------------------------- consumers
  const int tid = threadIdx.x;  // 0..255
  const int g = lane >> 2, t = lane & 3;
  const int cw = warp * 32 + 4 * g;          // first of this thread's 4 columns within the tile
  constexpr int rpf = 4 * SPF;               // word rows per flush group
  constexpr int subs = 4 / SPF;              // flush groups per unit
  const int upp = sk_units_per_piece(p.M);
  uint4* xr = reinterpret_cast<uint4*>(smem + kSkXOff);
  float* sums = reinterpret_cast<float*>(smem + kSkSumOff);
  // this thread's swizzled 16-byte column group in word row 4 j + t of its slab
  int woff[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) woff[j] = (4 * j + t) * 128 + ((g ^ ((4 * j + t) & 7)) << 4);
  constexpr uint32_t kBiasBits = BF16 ? 0x43000000u : 0x44800000u;  // fp32 bits of Mg = 128 / 1024
  constexpr uint32_t kZUnit = BF16 ? 65536u : 8192u;               // fp32 mantissa unit of 1.0 there

  // act-order indices of the first gather, loaded before waiting for the previous kernel
  int pre[2][8];
  int npre = 0;
  if (p.kperm) {
    const int tile0 = u0 / p.KB;
    const int npu0 = min(min(u1, (tile0 + 1) * p.KB), u0 + upp) - u0;
    const int kb0 = u0 - tile0 * p.KB;
    sk_load_idx(p, kb0, npu0 * 16, tid, pre[0]);
    sk_load_idx(p, kb0, npu0 * 16, tid + 256, pre[1]);
    npre = 2;
  }

  bool failed = false;
  int ring = 0;                 // unit index within the CTA's run (ring position)
  int dtile[2] = {0, 0}, dnseg[2] = {0, 0}, nd = 0;  // split tiles whose tickets this warp takes at the end
  float acc[MT][2][4];
  for (int su = u0; su < u1;) {
    const int tile = su / p.KB;
    const int se = min(u1, (tile + 1) * p.KB);
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

    for (int pu = su; pu < se; pu += upp) {
      const int pe = min(se, pu + upp);
      named_bar_sync(1, kSkWarps * 32);  // the previous piece's fragments are no longer read
      if (pu == u0) griddep_wait();     // x is written by the previous kernel in the stream
      sk_gather<BF16>(p, pu - tile * p.KB, pe - pu, rpf, xr, sums, tid, pre, pu == u0 ? npre : 0);
      named_bar_sync(1, kSkWarps * 32);
      if (pu == u0 && lane == 0) mbar_arrive(gathered);

      for (int u = pu; u < pe; ++u, ++ring) {
        if (failed) continue;
        const int s = ring % kSkDepth;
        // warp-uniform outcome: the lanes' bounded waits could disagree at the limit
        if (!__all_sync(0xffffffffu, mbar_wait_ns(&full[s], (ring / kSkDepth) & 1, abort_flag, kDevErrWFull,
                                                  p.wait_ns))) {
          failed = true;
          continue;
        }
        const int pi = u - pu;
        const uint4* xu = xr + pi * 16 * p.M;  // this unit's fragments
        const uint8_t* wst = smem + kSkWOff + s * kSkWBytes + warp * 2048;
        const uint8_t* sst = smem + kSkSOff + s * kSkSBytes;
        const uint8_t* zst = smem + kSkZOff + s * kSkZBytes;
        float cg[MT][2][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (j % SPF == 0) {
#pragma unroll
            for (int a = 0; a < MT; ++a)
#pragma unroll
              for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int c = 0; c < 4; ++c) cg[a][b][c] = 0.f;
          }
          const uint4 w = *reinterpret_cast<const uint4*>(wst + woff[j]);
          uint4 xv[MT];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int m = g + 8 * mt;
            xv[mt] = m < p.M ? xu[(4 * j + t) * p.M + m] : make_uint4(0u, 0u, 0u, 0u);
          }
          const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
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
#pragma unroll
            for (int beta = 0; beta < 2; ++beta) {
              const uint32_t a0[4] = {pr[2 * beta][0], pr[2 * beta + 1][0], pr[2 * beta][1], pr[2 * beta + 1][1]};
              const uint32_t a1[4] = {pr[2 * beta][2], pr[2 * beta + 1][2], pr[2 * beta][3], pr[2 * beta + 1][3]};
              mma_16816<BF16>(cg[mt][beta], a0, xv[mt].x, xv[mt].y);
              mma_16816<BF16>(cg[mt][beta], a1, xv[mt].z, xv[mt].w);
            }
          }
          if ((j + 1) % SPF == 0) {
            // flush group `sub` of this unit: scale row `sub` (groups < 128 rows) or 0
            const int sub = j / SPF;   // compile-time once the step loop is unrolled
            const int srow = SPF < 4 ? sub : 0;
            const uint2 sv = *reinterpret_cast<const uint2*>(sst + srow * (kSkCols * 2) + cw * 2);
            uint32_t zw = *reinterpret_cast<const uint32_t*>(zst + srow * (kSkCols / 2) + (cw / 8) * 4);
            if (p.v1) zw = ((zw & 0x77777777u) + 0x11111111u) ^ (zw & 0x88888888u);  // (z + 1) mod 16 per field
            float sc[4];
            if (p.s_dtype == kF16) {
              const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
              const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
              sc[0] = lo.x; sc[1] = lo.y; sc[2] = hi.x; sc[3] = hi.y;
            } else {
              sc[0] = __uint_as_float(sv.x << 16);
              sc[1] = __uint_as_float(sv.x & 0xFFFF0000u);
              sc[2] = __uint_as_float(sv.y << 16);
              sc[3] = __uint_as_float(sv.y & 0xFFFF0000u);
            }
            const int zsh = 4 * (cw & 7);
            float cz[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              cz[q] = sc[q] * __uint_as_float(((zw >> (zsh + 4 * q)) & 0xFu) * kZUnit + kBiasBits);  // s (Mg + z)
            const float* srow_x = sums + (pi * subs + sub) * p.M;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const int m0 = 8 * mt + 2 * t;
              const float x0 = m0 < p.M ? srow_x[m0] : 0.f;
              const float x1 = m0 + 1 < p.M ? srow_x[m0 + 1] : 0.f;
#pragma unroll
              for (int beta = 0; beta < 2; ++beta)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                  const int q = 2 * beta + (c >> 1);  // column 4g + q
                  acc[mt][beta][c] = fmaf(sc[q], cg[mt][beta][c], fmaf(-cz[q], (c & 1) ? x1 : x0, acc[mt][beta][c]));
                }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }

    // ---- segment end: this CTA's part of `tile` is complete (per warp: its 32 columns)
    const int c_first = (tile * p.KB) / p.upc;
    const int c_last = ((tile + 1) * p.KB - 1) / p.upc;
    const int nseg = c_last - c_first + 1;
    const int col = tile * kSkCols + cw;
    if (nseg == 1) {
      if (!failed && col < p.N) sk_write_out<BF16, MT>(p, acc, col, t);
    } else {
      if (!failed && col < p.N) {
        const long long slot = (long long)tile + blockIdx.x;
#pragma unroll
        for (int a = 0; a < MT; ++a)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int m = 8 * a + 2 * t + h;
            if (m < p.M)
              __stcg(reinterpret_cast<float4*>(p.ws + (slot * p.M + m) * kSkCols + cw),
                     make_float4(acc[a][0][h], acc[a][0][2 + h], acc[a][1][h], acc[a][1][2 + h]));
          }
      }
      if (nd < 2) {  // a run has at most two split tiles: its first and its last
        dtile[nd] = tile;
        dnseg[nd] = nseg;
        ++nd;
      }
    }
    su = se;
  }

  // ---- tickets of the split tiles (after the whole run: the partials above are long written)
  if (nd > 0) {
    __threadfence();
    __syncwarp();
    for (int d = 0; d < nd; ++d) {
      const int tile = dtile[d];
      unsigned prev = 0u;
      if (lane == 0) prev = atomicAdd(p.tickets + tile * kSkWarps + warp, failed ? 1u + kTicketFail : 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if ((prev & (kTicketFail - 1u)) != (unsigned)(dnseg[d] - 1)) continue;  // not the last segment
      if (lane == 0) p.tickets[tile * kSkWarps + warp] = 0u;                   // re-arm for the next launch
      if (prev >= kTicketFail || failed) continue;                            // a segment failed: no output
      __threadfence();
      const int col = tile * kSkCols + cw;
      if (col >= p.N) continue;
      const int c_first = (tile * p.KB) / p.upc;
      const int c_last = ((tile + 1) * p.KB - 1) / p.upc;
      float sum[MT][2][4];
#pragma unroll
      for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int m = 8 * a + 2 * t + h;
          float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if (m < p.M) {
            for (int c = c_first; c <= c_last; ++c) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(p.ws + (((long long)tile + c) * p.M + m) *
                                                                           kSkCols + cw));
              v4.x += v.x; v4.y += v.y; v4.z += v.z; v4.w += v.w;
            }
          }
          sum[a][0][h] = v4.x; sum[a][0][2 + h] = v4.y; sum[a][1][h] = v4.z; sum[a][1][2 + h] = v4.w;
        }
      sk_write_out<BF16, MT>(p, sum, col, t);
    }
  }
}

}  // namespace oc
